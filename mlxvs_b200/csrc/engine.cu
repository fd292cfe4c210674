// Host side of the exact k-NN engine: argument checks, scratch memory from
// the stream-ordered pool, TMA tensor maps, the choice between the exact
// one-pass fp16 path and the split-fp16 path, work decomposition and launches.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "engine.h"
#include "gemm_topk.cuh"
#include "gemm_topk_q.cuh"
#include "hamming.cuh"
#include "select.cuh"
#include "knn_kernels.cuh"

#ifndef MLXVS_B200_VERSION
#define MLXVS_B200_VERSION "0.16.1-b200"
#endif

namespace mlxvs_b200 {

namespace {

// Bounded waits inside the kernels give up after this long (no legitimate
// wait comes near it: stages turn over in microseconds).
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;

void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string("[mlxvs_b200] CUDA error: ") + cudaGetErrorString(e) +
                             " (" + what + ")");
  }
}
#define CK(x) check_cuda((x), #x)

void require(bool ok, const std::string& msg) {
  if (!ok) throw std::invalid_argument(msg);
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

struct DeviceInfo {
  int sms = 0;
  int max_smem = 0;
  uint32_t* err = nullptr;  // error word of the kernels' bounded waits
  size_t total_mem = 0;     // device memory in bytes
};

DeviceInfo& device_info() {
  static std::mutex mu;
  static DeviceInfo infos[64];
  static bool ready[64] = {};
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64)
    throw std::runtime_error("[mlxvs_b200] device ordinal " + std::to_string(dev) +
                             " is beyond the 64 devices this library tracks");
  std::lock_guard<std::mutex> guard(mu);
  DeviceInfo& info = infos[dev];
  if (!ready[dev]) {
    int major = 0, minor = 0;
    CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    CK(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (major != 10 || minor != 0)
      throw std::runtime_error("[mlxvs_b200] needs an sm_100 GPU (B200); device " +
                               std::to_string(dev) + " is sm_" + std::to_string(major) +
                               std::to_string(minor));
    CK(cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, dev));
    CK(cudaDeviceGetAttribute(&info.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    {
      size_t free_b = 0;
      CK(cudaMemGetInfo(&free_b, &info.total_mem));
    }
    CK(cudaMalloc(&info.err, 16));
    CK(cudaMemset(info.err, 0, 16));
    // keep freed scratch in this process's pool between calls
    cudaMemPool_t pool;
    CK(cudaDeviceGetDefaultMemPool(&pool, dev));
    uint64_t keep = UINT64_MAX;
    CK(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
    ready[dev] = true;
  }
  return info;
}

// ------------------------------------------------------------- profiling
// When enabled, every launch of the library's kernels is bracketed by CUDA
// events recorded on the launching stream; profile_read sums their device
// times per kernel name.  Off by default (benchmarks turn it on).
struct ProfRecord {
  const char* name;
  cudaEvent_t start, stop;
  double issued;  // tensor-core operations the launch issued (0: none)
};
std::mutex prof_mu;
bool prof_on = false;
std::vector<ProfRecord> prof_records;

struct ProfScope {
  const char* name;
  cudaStream_t s;
  cudaEvent_t start = nullptr, stop = nullptr;
  double issued = 0.0;
  ProfScope(const char* n, cudaStream_t st) : name(n), s(st) {
    bool on;
    {
      std::lock_guard<std::mutex> g(prof_mu);
      on = prof_on;
    }
    if (!on) return;
    CK(cudaEventCreate(&start));
    CK(cudaEventCreate(&stop));
    CK(cudaEventRecord(start, s));
  }
  ~ProfScope() {
    if (!start) return;
    cudaEventRecord(stop, s);
    std::lock_guard<std::mutex> g(prof_mu);
    prof_records.push_back({name, start, stop, issued});
  }
};

// A speculative launch is recorded as PROF_SPECULATIVE until the host knows
// whether it did the work: then as `kept_as`, or as PROF_SKIPPED (a launch
// that returned at entry, with no issued work).
constexpr const char* PROF_SPECULATIVE = "gemm_topk_speculative";
constexpr const char* PROF_SKIPPED = "gemm_topk_skipped";
void profile_resolve_speculative(const char* kept_as) {
  std::lock_guard<std::mutex> g(prof_mu);
  for (auto it = prof_records.rbegin(); it != prof_records.rend(); ++it) {
    if (std::strcmp(it->name, PROF_SPECULATIVE) != 0) continue;
    it->name = kept_as ? kept_as : PROF_SKIPPED;
    if (!kept_as) it->issued = 0.0;
    return;
  }
}

// The flags of a call's prep read back through pinned memory: one buffer and
// one event per (host thread, device), so a call waits for the copy alone
// while the kernels enqueued after it keep running.
// Pinned words the prep kernels' flags are copied into, on a stream of its
// own: the copy waits for the preps (event `prepped`) but the kernels queued
// after them on the caller's stream do not wait for the copy.
struct FlagMailbox {
  uint32_t* host = nullptr;
  cudaEvent_t ev = nullptr;
  cudaEvent_t prepped = nullptr;
  cudaStream_t side = nullptr;
};
FlagMailbox& flag_mailbox() {
  thread_local FlagMailbox boxes[64];
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64)
    throw std::runtime_error("[mlxvs_b200] device ordinal " + std::to_string(dev) +
                             " is beyond the 64 devices this library tracks");
  FlagMailbox& b = boxes[dev];
  if (b.host == nullptr) {
    CK(cudaHostAlloc(reinterpret_cast<void**>(&b.host), 64, cudaHostAllocDefault));
    CK(cudaEventCreateWithFlags(&b.ev, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&b.prepped, cudaEventDisableTiming));
    CK(cudaStreamCreateWithFlags(&b.side, cudaStreamNonBlocking));
  }
  return b;
}

// Scratch buffers of one call, returned to the pool in stream order.
struct Scratch {
  cudaStream_t s;
  std::vector<void*> ptrs;
  explicit Scratch(cudaStream_t st) : s(st) {}
  template <class T>
  T* alloc(size_t count) {
    void* p = nullptr;
    CK(cudaMallocAsync(&p, std::max<size_t>(count * sizeof(T), 256), s));
    ptrs.push_back(p);
    return static_cast<T*>(p);
  }
  ~Scratch() {
    for (void* p : ptrs) cudaFreeAsync(p, s);
  }
};

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) throw std::runtime_error("[mlxvs_b200] cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// 2-D fp16 tensor [rows, cols] (cols contiguous), tiles of box_cols x
// box_rows written to shared memory with the 128-byte swizzle (or the 32-byte
// one for the 16-column |b|^2 pieces).
CUtensorMap map_f16(const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols,
                    uint32_t box_rows,
                    CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("[mlxvs_b200] cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return m;
}

// Base ranges per query block: the fewest waves of units over the slots,
// each unit paying a fixed start cost of about `overhead` tiles.
int choose_splits(int qblocks, int tiles, int slots, double overhead, int max_splits) {
  int best = 1;
  double best_cost = 1e300;
  int limit = std::max(1, std::min(tiles, max_splits));
  for (int s = 1; s <= limit; ++s) {
    int64_t units = (int64_t)qblocks * s;
    int64_t waves = (units + slots - 1) / slots;
    double per_unit = std::ceil((double)tiles / s) + overhead;
    double cost = (double)waves * per_unit;
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

void launch_prep(const PrepParams& p, int sms, cudaStream_t s) {
  if (p.n_pad == 0) return;
  const int threads = 256;
  int64_t blocks = std::min<int64_t>((p.n_pad + 7) / 8, (int64_t)sms * 16);
  bool vec = p.d % 4 == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
  ProfScope prof("prep", s);
  if (vec && p.lo == nullptr && !p.cosine && p.d_pad <= 128) {
    const int64_t blocks4 = std::min<int64_t>((p.n_pad + 31) / 32, (int64_t)sms * 16);
    prep_rows4_kernel<<<(unsigned)blocks4, threads, 0, s>>>(p);
  } else if (vec && p.lo == nullptr && !p.cosine)
    prep_rows_vec4_kernel<false><<<(unsigned)blocks, threads, 0, s>>>(p);
  else if (vec)
    prep_rows_vec4_kernel<true><<<(unsigned)blocks, threads, 0, s>>>(p);
  else
    prep_rows_kernel<<<(unsigned)blocks, threads, 0, s>>>(p);
  CK(cudaGetLastError());
}

void launch_merge(const uint64_t* lists, int num_lists, int64_t list_rows, int64_t nq, int k,
                  int kind, const float* qq, uint64_t* out_keys, int32_t* ids, float* dist,
                  cudaStream_t s, float scale = 1.0f, const float* queries = nullptr,
                  int d = 0) {
  if (nq == 0) return;
  int64_t total = (int64_t)num_lists * k;
  if (merge_quad_fits(num_lists, k)) {
    ProfScope prof("merge", s);
    const unsigned blocks = (unsigned)((nq + 7) / 8);
    const size_t smem = (size_t)total * 8 * sizeof(uint64_t);
#define MLXVS_MERGE_QUAD(KR_)                                                              \
  merge_keys_quad_kernel<KR_><<<blocks, 32, smem, s>>>(lists, num_lists, list_rows, nq, k, \
                                                         kind, qq, out_keys, ids, dist, scale, \
                                                         queries, d)
    if (k <= 10)
      MLXVS_MERGE_QUAD(10);
    else if (k <= 16)
      MLXVS_MERGE_QUAD(16);
    else
      MLXVS_MERGE_QUAD(32);
#undef MLXVS_MERGE_QUAD
    CK(cudaGetLastError());
    return;
  }
  if (k <= 32 && total <= 32 * 32) {
    ProfScope prof("merge", s);
    const unsigned blocks = (unsigned)((nq + 7) / 8);
#define MLXVS_MERGE_WARP(M_)                                                            \
  merge_keys_warp_kernel<M_><<<blocks, 256, 0, s>>>(lists, num_lists, list_rows, nq, k, \
                                                     kind, qq, out_keys, ids, dist, scale)
    if (total <= 32 * 4)
      MLXVS_MERGE_WARP(4);
    else if (total <= 32 * 8)
      MLXVS_MERGE_WARP(8);
    else if (total <= 32 * 16)
      MLXVS_MERGE_WARP(16);
    else
      MLXVS_MERGE_WARP(32);
#undef MLXVS_MERGE_WARP
    CK(cudaGetLastError());
    return;
  }
  int cap = 2;
  while (cap < total && cap < MERGE_CAP) cap <<= 1;
  while (cap <= k) cap <<= 1;
  ProfScope prof("merge", s);
  merge_keys_kernel<<<(unsigned)nq, MERGE_THREADS, (size_t)cap * 8, s>>>(
      lists, num_lists, list_rows, nq, k, kind, qq, out_keys, ids, dist, cap, scale);
  CK(cudaGetLastError());
}

void launch_fill(int64_t count, int kind, int32_t* ids, float* dist, uint64_t* keys,
                 cudaStream_t s) {
  if (count == 0) return;
  unsigned blocks = (unsigned)std::min<int64_t>((count + 255) / 256, 4096);
  ProfScope prof("fill", s);
  fill_missing_kernel<<<blocks, 256, 0, s>>>(count, kind, ids, dist, keys);
  CK(cudaGetLastError());
}

struct GemmMaps {
  CUtensorMap a_hi, a_lo, b_hi, b_lo, b_x;
};

// The queued epilogue (gemm_topk_q.cuh) is the default wherever it applies;
// MLXVS_EPILOGUE=inline selects the inline one everywhere (for comparisons).
bool queued_epilogue_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("MLXVS_EPILOGUE");
    return !(e != nullptr && std::strcmp(e, "inline") == 0);
  }();
  return on;
}

// Ring depth and query-block placement of the queued kernel: at least
// `min_stages` stages (the inline kernel's depth for the same launch), the
// resident query block preferred, queues of QK_QD chunks.  Returns false
// when no such layout fits.
constexpr int QK_QD = 2;
bool pick_queued(const DeviceInfo& dev, int npa, int kchunks, int extra, int min_stages,
                 int* stages, int* a_stream, uint32_t* smem) {
  const uint32_t budget = (uint32_t)dev.max_smem - 1024u;
  for (int as : {0, 1}) {
    for (int st = 8; st >= min_stages; --st) {
      const QueuedSmem lay = queued_smem(npa, kchunks, st, as, extra, QK_QD);
      if (lay.total <= budget) {
        *stages = st;
        *a_stream = as;
        *smem = lay.total + 1024u;
        return true;
      }
    }
  }
  return false;
}

template <int QB, int NPASS, int CG, int NBM, int KR, int OP = 0, int MODE = 0>
void launch_gemm(const GemmMaps& m, const KnnGemmParams& p, int grid, uint32_t smem,
                 cudaStream_t s, const char* prof_name = nullptr) {
  ProfScope prof(prof_name ? prof_name
                           : (OP == 1 ? "hamming_mma" : (MODE == 1 ? "gemm_collect" : "gemm_topk")),
                 s);
  // every (query block, tile) pair runs 128 x 256 MMAs over the issued K:
  // NPASS fp16 products per 64-column chunk plus the K=16 |b|^2 block, or
  // 128 int8 columns per chunk
  const double k_issued = OP == 1 ? 128.0 * p.kchunks
                                  : (double)NPASS * GT_KCH * p.kchunks + 16.0 * p.extra;
  prof.issued = 2.0 * 128.0 * GT_BN * k_issued * (double)p.qblocks * (double)p.tiles;
  if constexpr (QB == QK_QB && CG == 2 && NPASS == 1 && (KR > 0 || MODE == 1)) {
    int st = 0, as = 0;
    uint32_t qsmem = 0;
    if (queued_epilogue_enabled() &&
        pick_queued(device_info(), 1, p.kchunks, p.extra, p.stages, &st, &as, &qsmem)) {
      KnnGemmParams pq = p;
      pq.stages = st;
      pq.a_stream = as;
      // the MMA loop unrolled over the K chunks for the common counts: 2 (fp16
      // rows of up to 128 values) and 8 (1024-bit codes as int8)
      constexpr int KQ = KR > 0 ? KR : 8;
      constexpr int KCH_FIXED = OP == 1 ? 8 : 2;
      auto kern = p.kchunks == KCH_FIXED
                      ? knn_gemm_topk_queued_kernel<NPASS, NBM, KQ, OP, MODE, QK_QD, KCH_FIXED>
                      : knn_gemm_topk_queued_kernel<NPASS, NBM, KQ, OP, MODE, QK_QD, 0>;
      CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)qsmem));
      kern<<<grid, QK_THREADS, qsmem, s>>>(m.a_hi, m.a_lo, m.b_hi, m.b_lo, m.b_x, pq);
      CK(cudaGetLastError());
      return;
    }
  }
  auto kern = knn_gemm_topk_kernel<QB, NPASS, CG, NBM, KR, OP, MODE>;
  CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  kern<<<grid, GemmLayout<QB, NPASS, CG>::THREADS, smem, s>>>(m.a_hi, m.a_lo, m.b_hi, m.b_lo,
                                                              m.b_x, p);
  CK(cudaGetLastError());
}

void check_rows(int64_t n, const char* what) {
  require(n >= 0 && n < (1LL << 31),
          std::string("[mlxvs::brute_force_knn] the number of ") + what +
              " must be in [0, 2^31).");
}

struct GemmShape {
  int qb, cg, kr, stages, a_stream;
};

// The fused kernel's shape, in order of preference: 128 queries per CTA
// with the 256 columns of a tile split over two warp groups (two lists per
// query, in registers for k <= 32 even with a shallower ring, else heaps in
// shared memory), then one warp group, then 64 .. 8 queries per CTA for
// large k (the MMA still computes 128 rows; the other lanes are unused);
// the query block resident in shared memory when it fits; the deepest ring
// that fits.
GemmShape choose_shape(const DeviceInfo& dev, int npa, int kchunks, int k, int extra, int nbm,
                       int want_stages) {
  const uint32_t budget = (uint32_t)dev.max_smem - 1024u;
  const int kr =
      k <= 8 ? 8 : (k <= 10 ? 10 : (k <= 12 ? 12 : (k <= 16 ? 16 : (k <= 32 ? 32 : 0))));
  struct Shape { int qb, cg, kr, min_st; };
  const Shape order[] = {{128, 2, kr, want_stages}, {128, 2, kr, 2},
                         {128, 2, 0, want_stages},  {128, 2, 0, 2},
                         {128, 1, 0, want_stages},  {128, 1, 0, 2},
                         {64, 1, 0, want_stages},   {64, 1, 0, 2},
                         {32, 1, 0, want_stages},   {32, 1, 0, 2},
                         {16, 1, 0, want_stages},   {16, 1, 0, 2},
                         {8, 1, 0, want_stages},    {8, 1, 0, 2}};
  for (const Shape& sh : order) {
    if (sh.cg == 2 && sh.kr == 0 && kr != 0) continue;  // the register list is the better form
    for (int as : {0, 1}) {
      for (int st = 8; st >= sh.min_st; --st) {
        if (gemm_smem(sh.qb, npa, sh.cg, kchunks, st, as, k, extra, sh.kr, nbm).total <= budget)
          return GemmShape{sh.qb, sh.cg, sh.kr, st, as};
      }
    }
  }
  throw std::runtime_error("[mlxvs_b200] no kernel shape fits shared memory");
}

// Launches the fused kernel of shape (qb, cg, kr) and operand passes for the
// given params (list mode, or collect mode for mode 1 with kr 8).
void launch_shape(const GemmMaps& maps, const KnnGemmParams& p, int qb, int cg, int kr,
                  bool exact, int nbm, int mode, uint32_t smem, int grid, cudaStream_t s) {
  bool launched = false;
#define MLXVS_GEMM_M(QB_, CG_, KR_, MODE_)                                   \
  if (!launched && qb == QB_ && cg == CG_ && kr == KR_ && mode == MODE_) {   \
    if (exact && nbm)                                                        \
      launch_gemm<QB_, 1, CG_, 1, KR_, 0, MODE_>(maps, p, grid, smem, s);    \
    else if (exact)                                                          \
      launch_gemm<QB_, 1, CG_, 0, KR_, 0, MODE_>(maps, p, grid, smem, s);    \
    else if (nbm)                                                            \
      launch_gemm<QB_, 3, CG_, 1, KR_, 0, MODE_>(maps, p, grid, smem, s);    \
    else                                                                     \
      launch_gemm<QB_, 3, CG_, 0, KR_, 0, MODE_>(maps, p, grid, smem, s);    \
    launched = true;                                                         \
  }
  MLXVS_GEMM_M(128, 2, 8, 1)
  MLXVS_GEMM_M(128, 2, 8, 0)
  MLXVS_GEMM_M(128, 2, 10, 0)
  MLXVS_GEMM_M(128, 2, 12, 0)
  MLXVS_GEMM_M(128, 2, 16, 0)
  MLXVS_GEMM_M(128, 2, 32, 0)
#undef MLXVS_GEMM_M
  require(launched, "[mlxvs_b200] no fused kernel for this shape");
}

// Large-k sizing: sample lists of LK_KG keys, 1 / LK_SAMPLE_DIV of the
// base tiles sampled (at least LK_MIN_TILES tiles per sample).
constexpr int LK_KG = 8;
constexpr int LK_SAMPLE_DIV = 4;
constexpr int LK_MIN_TILES = 16;
// Listed-sample floors (exact operands, k >= LK_LISTED_MIN_K): the best kp
// of every (c * k / kp)-th tile, so that some c * k rows of the base clear
// the floor, with (kp, c) = (16, 6) when that sample keeps at least
// LK_LISTED_MIN_TILES tiles, else (32, 4).  On rows in random order the
// number that clears it is about the stride times a Gamma(kp) variable,
// whose mean is c * k; it falls below k with probability about 2e-8 per
// query for (16, 6) and 1e-10 for (32, 4) (the select step then flags the
// query and the heap search runs instead); c grows with the number of
// queries so that a search needs that fallback with probability < 1e-3.  Measured on config 1 against
// the grouped floors: k = 17 -3 %, 24 -10 %, 32 -13 %, 64 -23 %, 100 -26 %,
// 128 -27 %, 256 -32 % per search.
struct ListedSample {
  int kp, c;  // sample list length, least collection factor
};

// The chance that fewer than k rows of a base in random order clear a
// listed floor of kp keys taken at stride c k / kp: P(Gamma(kp) < kp / c),
// i.e. P(Poisson(kp / c) >= kp).
double listed_underflow(int kp, int c) {
  const double lam = (double)kp / c;
  double term = std::exp(-lam);
  for (int i = 1; i <= kp; ++i) term *= lam / i;
  double tail = 0.0;
  for (int i = kp; i < kp + 64 && term > 0.0; ++i) {
    tail += term;
    term *= lam / (i + 1);
  }
  return tail;
}
constexpr ListedSample LK_LISTED[2] = {{16, 6}, {32, 4}};
constexpr int LK_LISTED_MIN_K = 17;
constexpr int LK_LISTED_MIN_TILES = 64;

// Exact search for k > 16 in three steps instead of one pass with long
// per-query lists (measured faster from k = 17 on):
//   A. a floor per query, one of two ways:
//      listed (exact operands, k >= LK_LISTED_MIN_K): the exact best kp of
//      a strided sample of the tiles, by the list kernel itself (shared
//      floors, inherited lists); its worst key, which about c * k rows
//      clear;
//      grouped (otherwise): over G = ceil(k / LK_KG) disjoint strided
//      samples, the exact best ceil(k / G) of each (units that do not share
//      lists or floors across samples); the smallest of the G worst keys has
//      G * ceil(k / G) >= k rows at or above it;
//   B. over the whole base, every candidate above that floor is kept
//      (collect mode, per (split, query, column group) buffers);
//   C. the best k of the kept candidates, then keys -> ids / distances.
// Returns false, having enqueued only harmless work, when a query kept more
// candidates than its buffers hold, or (listed floors) fewer than k: the
// caller then searches with heaps.
bool large_k_search(const GemmMaps& maps_in, const KnnGemmParams& p_in, bool exact, int nbm,
                    int npa, int kchunks, bool fold, const __half* q_hi, const __half* q_lo,
                    int64_t nq_pad, int d_pad, int mi, const float* qq, uint64_t* out_keys,
                    int32_t* ids, float* dist, float out_scale, Scratch& sc, cudaStream_t s,
                    RescoreParams* rescore = nullptr, float eps = 0.0f) {
  DeviceInfo& dev = device_info();
  const int k = p_in.k;
  const int tiles = p_in.tiles;
  // G samples: ceil(k / LK_KG), or up to 3 times that when its units fill the
  // SMs' waves much better (pass A takes about ceil(qblocks G / sms) / G of
  // its sample's time; more samples also mean a lower floor, so a larger G
  // must save a fifth of that)
  const int qb_count = (int)((p_in.nq + 127) / 128);
  const int g_min = (k + LK_KG - 1) / LK_KG;
  auto wave_time = [&](int g) {
    return (double)((qb_count * (int64_t)g + dev.sms - 1) / dev.sms) / g;
  };
  int G = g_min;
  double best_t = wave_time(g_min);
  for (int g = g_min + 1; g <= 3 * g_min; ++g) {
    const double t = wave_time(g);
    if (t < 0.8 * wave_time(g_min) && t < best_t * 0.999) {
      best_t = t;
      G = g;
    }
  }
  const int kg = (k + G - 1) / G;
  const int sample_tiles = std::max(LK_MIN_TILES * G, tiles / LK_SAMPLE_DIV);
  if ((k <= 16 && rescore == nullptr) || nq_pad % 128 != 0) return false;
  const int want = exact ? 4 : 2;
  const GemmShape sb = choose_shape(dev, npa, kchunks, 8, fold ? 1 : 0, nbm, want);
  if (sb.qb != 128 || sb.cg != 2 || sb.kr != 8) return false;
  // the listed sample: floors shared by the sample's splits and lists
  // inherited across them, so only the first wave of units starts cold
  int kp = 0, lstride = 0, ltiles = 0;
  for (const ListedSample& ls : LK_LISTED) {
    kp = ls.kp;
    // the factor grows with the queries until the chance that any of them
    // needs the fallback is under 1e-3 (config 3's 1M queries: 8 for kp 16)
    int c = ls.c;
    while (c < 16 && (double)p_in.nq * listed_underflow(kp, c) > 1e-3) ++c;
    lstride = std::max(2, c * k / kp);
    ltiles = tiles / lstride;
    if (ltiles >= LK_LISTED_MIN_TILES) break;
  }
  const GemmShape sl = choose_shape(dev, npa, kchunks, kp, fold ? 1 : 0, nbm, want);
  const bool listed = rescore == nullptr && k >= LK_LISTED_MIN_K &&
                      ltiles >= LK_LISTED_MIN_TILES && sl.qb == 128 && sl.cg == 2 &&
                      sl.kr == kp;
  const GemmShape sa = choose_shape(dev, npa, kchunks, kg, fold ? 1 : 0, nbm, want);
  if (!listed && (sample_tiles > tiles || sa.qb != 128 || sa.cg != 2 || sa.kr == 0))
    return false;
  const int64_t nq = p_in.nq;
  const int qblocks = (int)((nq + 127) / 128);
  GemmMaps maps = maps_in;
  maps.a_hi = map_f16(q_hi, d_pad, nq_pad, GT_KCH, 128);
  maps.a_lo = map_f16(q_lo ? q_lo : q_hi, d_pad, nq_pad, GT_KCH, 128);
  unsigned long long* floor = sc.alloc<unsigned long long>((size_t)nq_pad);
  int* done = sc.alloc<int>((size_t)qblocks);
  CK(cudaMemsetAsync(done, 0, (size_t)qblocks * 4, s));
  uint64_t* partial_a = nullptr;
  int32_t k_min = 0;  // candidates every query must keep (listed floors only)

  if (listed) {
    // A': the exact best kp of every lstride-th tile; its worst key is a
    // floor that some kp * lstride rows clear on average but, for k > kp,
    // not surely k of them: step C checks that
    KnnGemmParams pa = p_in;
    pa.qblocks = qblocks;
    pa.tiles = ltiles;
    pa.tile_stride = lstride;
    pa.splits = choose_splits(qblocks, ltiles, dev.sms, 3.0, 64);
    pa.units = qblocks * pa.splits;
    pa.k = kp;
    pa.stages = sl.stages;
    pa.a_stream = sl.a_stream;
    pa.no_inherit = 0;
    pa.gfloor_split_stride = 0;
    pa.gfloor = sc.alloc<unsigned long long>((size_t)nq_pad);
    CK(cudaMemsetAsync(pa.gfloor, 0, (size_t)nq_pad * 8, s));
    pa.partial = sc.alloc<uint64_t>((size_t)pa.splits * nq_pad * kp);
    pa.done = done;
    const GemmSmem lay =
        gemm_smem(128, npa, 2, kchunks, sl.stages, sl.a_stream, kp, fold, kp, nbm);
    launch_shape(maps, pa, 128, 2, kp, exact, nbm, 0, lay.total + 1024u,
                 std::min(pa.units, dev.sms), s);
    uint64_t* top = sc.alloc<uint64_t>((size_t)nq * kp);
    launch_merge(pa.partial, pa.splits, nq_pad, nq, kp, mi, nullptr, top, nullptr, nullptr, s);
    list_floor_kernel<<<(unsigned)((nq_pad + 255) / 256), 256, 0, s>>>(top, kp, nq, nq_pad,
                                                                       floor);
    CK(cudaGetLastError());
    partial_a = pa.partial;
    const int64_t avail = p_in.n_valid - (p_in.self_base >= 0 ? 1 : 0);
    k_min = (int32_t)std::min<int64_t>(k, avail);
  } else {
    // A: per-sample exact lists
    KnnGemmParams pa = p_in;
    pa.qblocks = qblocks;
    pa.tiles = sample_tiles;
    pa.splits = G;
    pa.units = qblocks * G;
    pa.k = kg;
    pa.stages = sa.stages;
    pa.a_stream = sa.a_stream;
    pa.tile_stride = tiles / sample_tiles;
    pa.no_inherit = 1;
    pa.gfloor_split_stride = nq_pad;
    pa.gfloor = sc.alloc<unsigned long long>((size_t)G * nq_pad);
    CK(cudaMemsetAsync(pa.gfloor, 0, (size_t)G * nq_pad * 8, s));
    pa.partial = sc.alloc<uint64_t>((size_t)G * nq_pad * kg);
    pa.done = done;
    {
      const GemmSmem lay = gemm_smem(128, npa, 2, kchunks, sa.stages, sa.a_stream, kg, fold, sa.kr,
                                     nbm);
      launch_shape(maps, pa, 128, 2, sa.kr, exact, nbm, 0, lay.total + 1024u,
                   std::min(pa.units, dev.sms), s);
    }
    sample_floor_kernel<<<(unsigned)((nq_pad + 255) / 256), 256, 0, s>>>(pa.partial, G, nq_pad, kg,
                                                                           nq, floor);
    CK(cudaGetLastError());
    if (rescore) {
      margin_floor_kernel<<<(unsigned)((nq + 255) / 256), 256, 0, s>>>(floor, nq, eps);
      CK(cudaGetLastError());
    }
    partial_a = pa.partial;
  }

  // B: every candidate above the floor
  KnnGemmParams pb = p_in;
  pb.qblocks = qblocks;
  pb.splits = choose_splits(qblocks, tiles, dev.sms, 3.0, 64);
  pb.units = qblocks * pb.splits;
  pb.k = 8;
  pb.stages = sb.stages;
  pb.a_stream = sb.a_stream;
  pb.tile_stride = 1;
  pb.no_inherit = 1;
  pb.gfloor = floor;
  pb.gfloor_split_stride = 0;
  pb.done = done;
  pb.partial = partial_a;  // not written in collect mode
  // some 10 k candidates per query are expected above the floor; room for
  // about five times that, spread over the splits and their two column
  // groups (one buffer each: `lists` per query)
  const int lists = pb.splits * 2;
  pb.collect_cap = (int)round_up(std::max<int64_t>(128, (int64_t)24 * k / pb.splits), 64);
  pb.collect = sc.alloc<uint64_t>((size_t)lists * nq_pad * pb.collect_cap);
  pb.collect_count = sc.alloc<int32_t>((size_t)lists * nq_pad);
  {
    const GemmSmem lay = gemm_smem(128, npa, 2, kchunks, sb.stages, sb.a_stream, 8, fold, 8, nbm);
    launch_shape(maps, pb, 128, 2, 8, exact, nbm, 1, lay.total + 1024u,
                 std::min(pb.units, dev.sms), s);
  }

  // (one fp16 pass) the kept candidates' exact scores
  if (rescore) {
    rescore->cand = pb.collect;
    rescore->count = pb.collect_count;
    rescore->splits = lists;
    rescore->nq = nq;
    rescore->nq_pad = nq_pad;
    rescore->cap = pb.collect_cap;
    const int64_t pairs = (int64_t)lists * nq;
    ProfScope prof("rescore", s);
    rescore_kernel<<<(unsigned)((pairs + 7) / 8), 256, 0, s>>>(*rescore);
    CK(cudaGetLastError());
  }

  // C: the best k of the kept candidates
  uint64_t* best = sc.alloc<uint64_t>((size_t)nq * k);
  int32_t* overflow = sc.alloc<int32_t>(1);
  CK(cudaMemsetAsync(overflow, 0, 4, s));
  {
    ProfScope prof("select_keys", s);
    select_keys_kernel<<<(unsigned)nq, TOPK_THREADS, 0, s>>>(
        pb.collect, pb.collect_count, lists, nq_pad, pb.collect_cap, nq, k, k_min, best,
        overflow);
    CK(cudaGetLastError());
  }
  int32_t h_overflow = 0;
  CK(cudaMemcpyAsync(&h_overflow, overflow, 4, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  if (h_overflow) return false;
  launch_merge(best, 1, nq, nq, k, mi, qq, out_keys, ids, dist, s, out_scale);
  return true;
}

// Inexact float operands: one fp16 pass with a margin and exact rescoring
// (large_k_search in its rescoring form).  b_hi / q_hi hold the scaled
// fp16 operands, nb the scaled |b|^2 (L2), qq the unscaled |q|^2 (L2).
bool approx_search(const float* base, int64_t n, const float* queries, int64_t nq, int d, int k,
                   int mi, int64_t id_offset, int64_t self_base, const __half* b_hi,
                   const __half* q_hi, const float* nb, const float* qq, int64_t n_pad,
                   int64_t nq_pad, int d_pad, int kchunks, int nbm, float eps,
                   uint64_t* out_keys, int32_t* ids, float* dist, Scratch& sc, cudaStream_t s) {
  DeviceInfo& dev = device_info();
  if (!(eps < INFINITY)) return false;
  GemmMaps maps;
  maps.a_hi = map_f16(q_hi, d_pad, nq_pad, GT_KCH, 128);
  maps.a_lo = maps.a_hi;
  maps.b_hi = map_f16(b_hi, d_pad, n_pad, GT_KCH, GT_BN);
  maps.b_lo = maps.b_hi;
  maps.b_x = maps.b_hi;
  KnnGemmParams p{};
  p.qblocks = (int)((nq + 127) / 128);
  p.tiles = (int)(n_pad / GT_BN);
  p.kchunks = kchunks;
  p.k = k;
  p.extra = 0;
  p.n_valid = n;
  p.nq = nq;
  p.nq_pad = nq_pad;
  p.id_offset = id_offset;
  p.nb = nb;
  p.self_base = self_base;
  p.tile_stride = 1;
  p.err = dev.err;
  p.wait_ns = WAIT_LIMIT_NS;
  RescoreParams rs{};
  rs.base = base;
  rs.queries = queries;
  rs.n = n;
  rs.d = d;
  rs.id_offset = id_offset;
  rs.metric = mi;
  return large_k_search(maps, p, true, nbm, 1, kchunks, false, q_hi, nullptr, nq_pad, d_pad, mi,
                        qq, out_keys, ids, dist, 1.0f, sc, s, &rs, eps);
}

// Scratch, tensor maps and parameters of one fused launch over (query block,
// base range) units: npa operand planes (1: the inputs exactly in fp16, 2:
// split hi / lo), fold: -|b|^2 rides in the MMA as one more K step, nbm: the
// accumulator is the score (else the epilogue subtracts nb).
struct FusedPlan {
  GemmShape shape;
  GemmMaps maps;
  KnnGemmParams p;
  uint64_t* partial;
  int grid;
  uint32_t smem;
};

// The start cost of a unit in tiles, for choose_splits (a compile-time
// constant so that other values can be built and timed).
#ifndef MLXVS_UNIT_OVERHEAD_TILES
#define MLXVS_UNIT_OVERHEAD_TILES 3.0
#endif

FusedPlan plan_fused(const DeviceInfo& dev, int npa, bool fold, int nbm, int kchunks, int k,
                     int64_t nq, int64_t n_pad, int64_t nq_pad, int d_pad, const __half* q_hi,
                     const __half* q_lo, const __half* b_hi, const __half* b_lo,
                     const __half* b_x, const float* nb, int64_t n, int64_t id_offset,
                     int64_t self_base, Scratch& sc, cudaStream_t s) {
  FusedPlan f{};
  f.shape = choose_shape(dev, npa, kchunks, k, fold ? 1 : 0, nbm, npa == 1 ? 4 : 2);
  const int QB = f.shape.qb;
  const int qblocks = (int)((nq + QB - 1) / QB);
  const int tiles = (int)(n_pad / GT_BN);
  const int splits = choose_splits(qblocks, tiles, dev.sms, MLXVS_UNIT_OVERHEAD_TILES, 64);
  const int units = qblocks * splits;

  f.partial = sc.alloc<uint64_t>((size_t)splits * nq_pad * k);
  unsigned long long* gfloor = sc.alloc<unsigned long long>((size_t)nq_pad);
  CK(cudaMemsetAsync(gfloor, 0, (size_t)nq_pad * 8, s));
  int* done = sc.alloc<int>((size_t)qblocks);
  CK(cudaMemsetAsync(done, 0, (size_t)qblocks * 4, s));

  f.maps.a_hi = map_f16(q_hi, d_pad, nq_pad, GT_KCH, QB);
  f.maps.a_lo = map_f16(q_lo ? q_lo : q_hi, d_pad, nq_pad, GT_KCH, QB);
  f.maps.b_hi = map_f16(b_hi, d_pad, n_pad, GT_KCH, GT_BN);
  f.maps.b_lo = map_f16(b_lo ? b_lo : b_hi, d_pad, n_pad, GT_KCH, GT_BN);
  f.maps.b_x = fold ? map_f16(b_x, 16, n_pad, 16, GT_BN, CU_TENSOR_MAP_SWIZZLE_32B) : f.maps.b_hi;

  KnnGemmParams& p = f.p;
  p.qblocks = qblocks;
  p.tiles = tiles;
  p.splits = splits;
  p.units = units;
  p.kchunks = kchunks;
  p.k = k;
  p.stages = f.shape.stages;
  p.a_stream = f.shape.a_stream;
  p.extra = fold ? 1 : 0;
  p.n_valid = n;
  p.nq = nq;
  p.nq_pad = nq_pad;
  p.id_offset = id_offset;
  p.nb = nb;
  p.partial = f.partial;
  p.gfloor = gfloor;
  p.done = done;
  p.self_base = self_base;
  p.tile_stride = 1;
  p.err = dev.err;
  p.wait_ns = WAIT_LIMIT_NS;
  const GemmSmem lay = gemm_smem(QB, npa, f.shape.cg, kchunks, f.shape.stages, f.shape.a_stream,
                                 k, fold, f.shape.kr, nbm);
  f.smem = lay.total + 1024u;
  f.grid = std::min(units, dev.sms);
  return f;
}

// The fused kernel of a plan: exact (one fp16 pass) or three split passes.
void launch_fused(const FusedPlan& f, bool exact, int nbm, cudaStream_t s,
                  const char* prof_name = nullptr) {
  const int QB = f.shape.qb, CG = f.shape.cg, KR = f.shape.kr;
#define MLXVS_GEMM(QB_, CG_, KR_)                                                  \
  if (QB == QB_ && CG == CG_ && KR == KR_) {                                       \
    if (exact && nbm)                                                            \
      launch_gemm<QB_, 1, CG_, 1, KR_>(f.maps, f.p, f.grid, f.smem, s, prof_name); \
    else if (exact)                                                              \
      launch_gemm<QB_, 1, CG_, 0, KR_>(f.maps, f.p, f.grid, f.smem, s, prof_name); \
    else if (nbm)                                                                \
      launch_gemm<QB_, 3, CG_, 1, KR_>(f.maps, f.p, f.grid, f.smem, s, prof_name); \
    else                                                                         \
      launch_gemm<QB_, 3, CG_, 0, KR_>(f.maps, f.p, f.grid, f.smem, s, prof_name); \
  }
  MLXVS_GEMM(128, 2, 8)
  MLXVS_GEMM(128, 2, 10)
  MLXVS_GEMM(128, 2, 12)
  MLXVS_GEMM(128, 2, 16)
  MLXVS_GEMM(128, 2, 32)
  MLXVS_GEMM(128, 2, 0)
  MLXVS_GEMM(128, 1, 0)
  MLXVS_GEMM(64, 1, 0)
  MLXVS_GEMM(32, 1, 0)
  MLXVS_GEMM(16, 1, 0)
  MLXVS_GEMM(8, 1, 0)
#undef MLXVS_GEMM
}

// The exact k-NN of queries among base: keys [nq, k] (out_keys) and / or ids
// and distances.  The per-call flow:
//   1. prep: fp32 -> fp16 operand rows (2q for L2), |b|^2, |q|^2, and whether
//      every value is exactly an fp16 (one host sync to read the flags);
//   2. if not: split-fp16 operands hi / lo with power-of-two scales;
//   3. the fused GEMM + top-k kernel over (query block, base range) units;
//   4. merge of the units' lists into the k best, then distances.
void knn_core(const float* base, int64_t n, const float* queries, int64_t nq, int d, int k,
              Metric metric, int64_t id_offset, uint64_t* out_keys, int32_t* ids, float* dist,
              cudaStream_t s, int64_t self_base = -1) {
  require(k >= 1 && k <= 256, "[mlxvs::brute_force_knn] k must be in [1, 256].");
  require(d >= 1, "[mlxvs::brute_force_knn] the dimension must be at least 1.");
  check_rows(n, "base rows");
  check_rows(nq, "queries");
  const int mi = static_cast<int>(metric);
  require(mi >= 0 && mi <= 2, "[mlxvs::brute_force_knn] unknown metric.");
  require(id_offset >= 0 && id_offset + n <= (1LL << 31),
          "[mlxvs::brute_force_knn] ids must fit in int32.");
  DeviceInfo& dev = device_info();
  if (nq == 0) return;
  if (n == 0) {
    launch_fill(nq * k, mi, ids, dist, out_keys, s);
    return;
  }
  require(base != nullptr && queries != nullptr, "[mlxvs::brute_force_knn] null input.");
  const bool l2 = metric == Metric::L2;
  const bool cosine = metric == Metric::Cosine;
  const int d_pad = (int)round_up(d, GT_KCH);
  const int kchunks = d_pad / GT_KCH;
  const int64_t n_pad = round_up(n, GT_BN);
  const int64_t nq_pad = round_up(nq, 128);

  Scratch sc(s);
  __half* b_hi = sc.alloc<__half>((size_t)n_pad * d_pad);
  __half* q_hi = sc.alloc<__half>((size_t)nq_pad * d_pad);
  float* nb = sc.alloc<float>((size_t)n_pad);
  float* qq = l2 ? sc.alloc<float>((size_t)nq_pad) : nullptr;
  // |b|^2 as fp16 pieces for the extra K step (L2)
  __half* b_x = l2 ? sc.alloc<__half>((size_t)n_pad * 16) : nullptr;
  // flags: base inexact, base max |x|, query inexact, query max |x|, base
  // |b|^2 not foldable
  uint32_t* flags = sc.alloc<uint32_t>(8);
  CK(cudaMemsetAsync(flags, 0, 32, s));

  // flags[5], flags[6]: the largest squared row norm of the base and query
  // operands (before scaling), for the error bound of one fp16 pass
  PrepParams pb{base, n, n_pad, d, d_pad, cosine ? 1 : 0, 1.0f, 1.0f, b_hi, nullptr,
                nb, l2 ? 1.0f : 0.0f, INFINITY, flags, b_x, flags + 4, flags + 5};
  PrepParams pq{queries, nq, nq_pad, d, d_pad, cosine ? 1 : 0, l2 ? 2.0f : 1.0f, 1.0f, q_hi,
                nullptr, qq, 1.0f, 0.0f, flags + 2, nullptr, nullptr, flags + 6};
  launch_prep(pb, dev.sms, s);
  launch_prep(pq, dev.sms, s);
  FlagMailbox& mb = flag_mailbox();
  CK(cudaEventRecord(mb.prepped, s));
  CK(cudaStreamWaitEvent(mb.side, mb.prepped, 0));
  CK(cudaMemcpyAsync(mb.host, flags, 32, cudaMemcpyDeviceToHost, mb.side));
  CK(cudaEventRecord(mb.ev, mb.side));
  // k <= 16 (register lists), L2 or inner product: the one-pass search on
  // exact operands (for L2 with -|b|^2 in the MMA) is launched before the
  // flags are read, so the GPU does not wait for the host; its CTAs return
  // at entry when the flags rule it out.  Cosine rows are unit rows, hardly
  // ever exact in fp16, so they do not speculate.
  const bool spec = k <= 16 && !cosine;
  FusedPlan sp{};
  if (spec) {
    sp = plan_fused(dev, 1, l2, 1, kchunks, k, nq, n_pad, nq_pad, d_pad, q_hi, nullptr, b_hi,
                    nullptr, b_x, nb, n, id_offset, self_base, sc, s);
    sp.p.skip_if = flags;
    launch_fused(sp, true, 1, s, PROF_SPECULATIVE);
  }
  CK(cudaEventSynchronize(mb.ev));
  uint32_t hflags[8];
  std::memcpy(hflags, mb.host, 32);
  const bool exact = hflags[0] == 0 && hflags[2] == 0;
  // L2 on exact operands with integer |b|^2 < 2^31: -|b|^2 rides in the MMA
  // and the epilogue reads scores straight from the accumulator
  const bool fold = l2 && exact && hflags[4] == 0;
  const int nbm = (!l2 || fold) ? 1 : 0;
  if (spec) {
    // the device made the same decision from the same words
    const bool kept = exact && (fold || !l2);
    profile_resolve_speculative(kept ? "gemm_topk" : nullptr);
    if (kept) {
      launch_merge(sp.partial, sp.p.splits, nq_pad, nq, k, mi, qq, out_keys, ids, dist, s);
      return;
    }
  }

  __half* b_lo = nullptr;
  __half* q_lo = nullptr;
  float out_scale = 1.0f;
  if (!exact) {
    float amax_b, amax_q;
    std::memcpy(&amax_b, &hflags[1], 4);
    std::memcpy(&amax_q, &hflags[3], 4);
    // power-of-two scales putting each operand's largest |value| in
    // [2^14, 2^15): the fp16 hi part keeps 11 bits, lo the next 11
    auto scale_exp = [](float amax) {
      if (!(amax > 0.0f) || !std::isfinite(amax)) return 0;
      return std::max(-60, std::min(60, 14 - std::ilogb(amax)));
    };
    const int eb = scale_exp(amax_b), eq = scale_exp(amax_q);
    if (n_pad / GT_BN >= 64) {
      // one fp16 pass of the scaled operands (hi only), every candidate
      // within twice its error bound of a sampled floor kept, then exact
      // float32 scores; the three-pass split below when buffers overflow
      float nb2, nq2;
      std::memcpy(&nb2, &hflags[5], 4);
      std::memcpy(&nq2, &hflags[6], 4);
      // |fp16 dot - exact dot| <= (2u + u^2 + (d + 16) 2^-24) |a| |b| (rounding
      // of both operands, u = 2^-11, and of the fp32 accumulation) plus
      // 2^-25 sqrt(d) (|a| + |b|) for operands in fp16's subnormal range; L2
      // adds the rounding of "dot - |b|^2"; doubled for safety.  In the
      // operands' scaled units (scales 2^xb, 2^xq).
      auto bound = [&](int xb, int xq) {
        const double na = std::sqrt((double)nq2) * 1.001 * std::ldexp(1.0, xq);
        const double nbn = std::sqrt((double)nb2) * 1.001 * std::ldexp(1.0, xb);
        const double u = std::ldexp(1.0, -11);
        double e = (2 * u + u * u + (d + 16) * std::ldexp(1.0, -24)) * na * nbn +
                   std::ldexp(1.0, -25) * std::sqrt((double)d) * (na + nbn);
        if (l2)
          e += std::ldexp(1.0, -23) * (na * nbn + (double)nb2 * 1.001 * std::ldexp(1.0, xb + xq));
        return 2.0 * e;
      };
      // The first prep pass wrote the operands at scale 1 (and |b|^2, |q|^2
      // for it).  Keep them when they are clear of fp16's overflow and the
      // bound at scale 1 is within 1 % of the bound at the best scales, in
      // unscaled units (unit rows: the subnormal term is about 2e-6 of the
      // rounding term), which saves a second pass over the base.
      const double qmul = l2 ? 2.0 : 1.0;
      const bool keep = amax_b < 16384.0f && qmul * amax_q < 16384.0 &&
                        bound(0, 0) <= 1.01 * bound(eb, eq) * std::ldexp(1.0, -(eb + eq));
      // the one-pass scales (the split passes below always use eb, eq)
      const int xb = keep ? 0 : eb, xq = keep ? 0 : eq;
      if (!keep) {
        const float sb = std::ldexp(1.0f, eb), sq = std::ldexp(1.0f, eq);
        PrepParams pb1{base, n, n_pad, d, d_pad, cosine ? 1 : 0, 1.0f, sb, b_hi, nullptr,
                       nb, l2 ? std::ldexp(1.0f, eb + eq) : 0.0f, INFINITY, nullptr, nullptr,
                       nullptr};
        PrepParams pq1{queries, nq, nq_pad, d, d_pad, cosine ? 1 : 0, l2 ? 2.0f : 1.0f, sq,
                       q_hi, nullptr, nullptr, 0.0f, 0.0f, nullptr, nullptr, nullptr};
        launch_prep(pb1, dev.sms, s);
        launch_prep(pq1, dev.sms, s);
      }
      const float eps = (float)bound(xb, xq);
      if (approx_search(base, n, queries, nq, d, k, mi, id_offset, self_base, b_hi, q_hi, nb, qq,
                        n_pad, nq_pad, d_pad, kchunks, l2 ? 0 : 1, eps, out_keys, ids, dist, sc,
                        s))
        return;
    }
    const float sb = std::ldexp(1.0f, eb), sq = std::ldexp(1.0f, eq);
    b_lo = sc.alloc<__half>((size_t)n_pad * d_pad);
    q_lo = sc.alloc<__half>((size_t)nq_pad * d_pad);
    PrepParams pb2{base, n, n_pad, d, d_pad, cosine ? 1 : 0, 1.0f, sb, b_hi, b_lo,
                   nb, l2 ? std::ldexp(1.0f, eb + eq) : 0.0f, INFINITY, nullptr, nullptr, nullptr};
    PrepParams pq2{queries, nq, nq_pad, d, d_pad, cosine ? 1 : 0, l2 ? 2.0f : 1.0f, sq, q_hi,
                   q_lo, nullptr, 0.0f, 0.0f, nullptr, nullptr, nullptr};
    launch_prep(pb2, dev.sms, s);
    launch_prep(pq2, dev.sms, s);
    out_scale = std::ldexp(1.0f, -(eb + eq));
  }

  const int npa = exact ? 1 : 2;
  FusedPlan f = plan_fused(dev, npa, fold, nbm, kchunks, k, nq, n_pad, nq_pad, d_pad, q_hi, q_lo,
                           b_hi, b_lo, b_x, nb, n, id_offset, self_base, sc, s);
  if (k > 16 && large_k_search(f.maps, f.p, exact, nbm, npa, kchunks, fold, q_hi, q_lo, nq_pad,
                                d_pad, mi, qq, out_keys, ids, dist, out_scale, sc, s))
    return;
  launch_fused(f, exact, nbm, s);
  launch_merge(f.partial, f.p.splits, nq_pad, nq, k, mi, qq, out_keys, ids, dist, s, out_scale);
}

// ------------------------------------------------------------------ Hamming

struct HammingOut {
  uint64_t* keys;
  int32_t* ids;
  float* dist;
};

// Picks the ring depth and split count of one kernel shape from its
// occupancy, then launches the scan and the merge of its lists.
template <int V, int QH>
void launch_hamming_t(HammingParams p, const DeviceInfo& dev, Scratch& sc, const HammingOut& out,
                      cudaStream_t s) {
  auto kern = hamming_topk_kernel<V, QH>;
  int stages = 4;
  uint32_t smem = hamming_smem_bytes(V, QH, p.k, stages);
  while (smem > (uint32_t)dev.max_smem && stages > 2)
    smem = hamming_smem_bytes(V, QH, p.k, --stages);
  if (smem > (uint32_t)dev.max_smem)
    throw std::runtime_error("[mlxvs_b200] hamming: no kernel shape fits shared memory");
  p.stages = stages;
  CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 1;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, QH + 32, smem));
  const int slots = dev.sms * std::max(per_sm, 1);
  p.splits = choose_splits(p.qblocks, p.tiles, slots, 2.0, 64);
  p.units = p.qblocks * p.splits;
  p.partial = sc.alloc<uint64_t>((size_t)p.splits * p.nq_pad * p.k);
  const int grid = std::min(p.units, slots);
  {
    ProfScope prof("hamming_topk", s);
    kern<<<grid, QH + 32, smem, s>>>(p);
    CK(cudaGetLastError());
  }
  launch_merge(p.partial, p.splits, p.nq_pad, p.nq, p.k, KIND_HAMMING, nullptr, out.keys, out.ids,
               out.dist, s);
}

template <int V>
void launch_hamming_v(const HammingParams& p, int QH, const DeviceInfo& dev, Scratch& sc,
                      const HammingOut& out, cudaStream_t s) {
  if constexpr (V <= 16) {
    if (QH == 256) return launch_hamming_t<V, 256>(p, dev, sc, out, s);
  }
  if (QH == 128) return launch_hamming_t<V, 128>(p, dev, sc, out, s);
  return launch_hamming_t<V, 64>(p, dev, sc, out, s);
}

// Hamming k-NN on the tensor cores: codes unpacked to +-1 int8 rows, one
// kind::i8 MMA pass of the fused kernel (s32 dots, exact), scores
// -(bits - dot) / 2 = -distance, so the keys equal those of the popcount
// kernel.  Returns false (nothing enqueued) when the unpacked rows would
// take more than 40 % of the device's memory.
bool hamming_mma(const uint8_t* rows, int64_t n, const uint8_t* queries, int64_t nq, int bytes,
                 int k, int64_t id_offset, uint64_t* out_keys, int32_t* ids, float* dist,
                 cudaStream_t s) {
  DeviceInfo& dev = device_info();
  const int bits = bytes * 8;
  const int d_pad = (int)round_up(bits, 128);  // one 128-byte K chunk per 128 bits
  const int kchunks = d_pad / 128;
  const int64_t n_pad = round_up(n, GT_BN);
  const int64_t nq_pad = round_up(nq, 128);
  // (the device's total memory, read once: a query of the free memory on
  // every call would cost a synchronization)
  if ((double)(n_pad + nq_pad) * d_pad > 0.4 * (double)dev.total_mem) return false;
  const GemmShape sh = choose_shape(dev, 1, kchunks, k, 0, 1, 4);
  Scratch sc(s);
  int8_t* b8 = sc.alloc<int8_t>((size_t)n_pad * d_pad);
  int8_t* q8 = sc.alloc<int8_t>((size_t)nq_pad * d_pad);
  {
    ProfScope prof("prep", s);
    const int64_t gb = std::min<int64_t>((n_pad * (d_pad / 16) + 255) / 256, (int64_t)dev.sms * 32);
    hamming_unpack_kernel<<<(unsigned)gb, 256, 0, s>>>(rows, n, n_pad, bytes, d_pad, b8);
    CK(cudaGetLastError());
    const int64_t gq = std::min<int64_t>((nq_pad * (d_pad / 16) + 255) / 256, (int64_t)dev.sms * 32);
    hamming_unpack_kernel<<<(unsigned)gq, 256, 0, s>>>(queries, nq, nq_pad, bytes, d_pad, q8);
    CK(cudaGetLastError());
  }
  const int qblocks = (int)((nq + sh.qb - 1) / sh.qb);
  const int tiles = (int)(n_pad / GT_BN);
  const int splits = choose_splits(qblocks, tiles, dev.sms, 3.0, 64);
  uint64_t* partial = sc.alloc<uint64_t>((size_t)splits * nq_pad * k);
  unsigned long long* gfloor = sc.alloc<unsigned long long>((size_t)nq_pad);
  CK(cudaMemsetAsync(gfloor, 0, (size_t)nq_pad * 8, s));
  int* done = sc.alloc<int>((size_t)qblocks);
  CK(cudaMemsetAsync(done, 0, (size_t)qblocks * 4, s));
  // int8 rows through the fp16 tensor maps: d_pad bytes = d_pad / 2 halves
  GemmMaps maps;
  maps.a_hi = map_f16(reinterpret_cast<__half*>(q8), d_pad / 2, nq_pad, GT_KCH, sh.qb);
  maps.b_hi = map_f16(reinterpret_cast<__half*>(b8), d_pad / 2, n_pad, GT_KCH, GT_BN);
  maps.a_lo = maps.a_hi;
  maps.b_lo = maps.b_hi;
  maps.b_x = maps.b_hi;
  KnnGemmParams p{};
  p.qblocks = qblocks;
  p.tiles = tiles;
  p.splits = splits;
  p.units = qblocks * splits;
  p.kchunks = kchunks;
  p.k = k;
  p.stages = sh.stages;
  p.a_stream = sh.a_stream;
  p.extra = 0;
  p.n_valid = n;
  p.nq = nq;
  p.nq_pad = nq_pad;
  p.id_offset = id_offset;
  p.nb = nullptr;
  p.partial = partial;
  p.gfloor = gfloor;
  p.done = done;
  p.dot_offset = -0.5f * (float)bits;
  p.self_base = -1;
  p.tile_stride = 1;
  p.err = dev.err;
  p.wait_ns = WAIT_LIMIT_NS;
  const GemmSmem lay = gemm_smem(sh.qb, 1, sh.cg, kchunks, sh.stages, sh.a_stream, k, 0, sh.kr, 1);
  const uint32_t smem = lay.total + 1024u;
  const int grid = std::min(p.units, dev.sms);
  bool launched = false;
#define MLXVS_HGEMM(QB_, CG_, KR_)                                      \
  if (!launched && sh.qb == QB_ && sh.cg == CG_ && sh.kr == KR_) {     \
    launch_gemm<QB_, 1, CG_, 1, KR_, 1>(maps, p, grid, smem, s);       \
    launched = true;                                                   \
  }
  MLXVS_HGEMM(128, 2, 8)
  MLXVS_HGEMM(128, 2, 10)
  MLXVS_HGEMM(128, 2, 12)
  MLXVS_HGEMM(128, 2, 16)
  MLXVS_HGEMM(128, 2, 32)
  MLXVS_HGEMM(128, 2, 0)
  MLXVS_HGEMM(128, 1, 0)
  MLXVS_HGEMM(64, 1, 0)
  MLXVS_HGEMM(32, 1, 0)
  MLXVS_HGEMM(16, 1, 0)
  MLXVS_HGEMM(8, 1, 0)
#undef MLXVS_HGEMM
  require(launched, "[mlxvs_b200] hamming: no tensor-core kernel for this shape");
  launch_merge(partial, splits, nq_pad, nq, k, KIND_HAMMING, nullptr, out_keys, ids, dist, s);
  return true;
}

void hamming_core(const uint8_t* rows, int64_t n, const uint8_t* queries, int64_t nq, int bytes,
                  int k, int64_t id_offset, uint64_t* out_keys, int32_t* ids, float* dist,
                  cudaStream_t s) {
  require(k >= 1 && k <= 256, "[mlxvs::hamming_knn] k must be in [1, 256].");
  require(bytes >= 1, "[mlxvs::hamming_knn] rows must be bit-packed uint8 [n, bytes].");
  require(bytes <= 512, "[mlxvs::hamming_knn] codes longer than 4096 bits are not supported.");
  require(n >= 0 && n < (1LL << 31),
          "[mlxvs::hamming_knn] the number of rows must be in [0, 2^31).");
  require(nq >= 0 && nq < (1LL << 31),
          "[mlxvs::hamming_knn] the number of queries must be in [0, 2^31).");
  require(id_offset >= 0 && id_offset + n <= (1LL << 31),
          "[mlxvs::hamming_knn] ids must fit in int32.");
  DeviceInfo& dev = device_info();
  if (nq == 0) return;
  if (n == 0) {
    launch_fill(nq * k, KIND_HAMMING, ids, dist, out_keys, s);
    return;
  }
  require(rows != nullptr && queries != nullptr, "[mlxvs::hamming_knn] null input.");
  if (hamming_mma(rows, n, queries, nq, bytes, k, id_offset, out_keys, ids, dist, s)) return;
  int V = 1;
  while (V * 16 < bytes) V <<= 1;
  const int row_bytes = 16 * V;
  Scratch sc(s);
  const uint8_t* r = rows;
  const uint8_t* qv = queries;
  // codes zero padded to 16 V bytes (zeros XOR zeros add nothing) when the
  // caller's layout is not already that, or not 16-byte aligned
  if (row_bytes != bytes || (reinterpret_cast<uintptr_t>(rows) & 15)) {
    uint8_t* pr = sc.alloc<uint8_t>((size_t)n * row_bytes);
    CK(cudaMemsetAsync(pr, 0, (size_t)n * row_bytes, s));
    CK(cudaMemcpy2DAsync(pr, row_bytes, rows, bytes, bytes, n, cudaMemcpyDeviceToDevice, s));
    r = pr;
  }
  if (row_bytes != bytes || (reinterpret_cast<uintptr_t>(queries) & 15)) {
    uint8_t* pq = sc.alloc<uint8_t>((size_t)nq * row_bytes);
    CK(cudaMemsetAsync(pq, 0, (size_t)nq * row_bytes, s));
    CK(cudaMemcpy2DAsync(pq, row_bytes, queries, bytes, bytes, nq, cudaMemcpyDeviceToDevice, s));
    qv = pq;
  }
  // queries per CTA: 256 while the heaps stay within 64 KB (two CTAs per SM)
  int QH = 256;
  while (QH > 64 && (uint32_t)QH * k * 8u > 64u * 1024u) QH >>= 1;
  if (V > 16 && QH > 128) QH = 128;
  const int64_t nq_pad = round_up(nq, QH);
  HammingParams p{};
  p.rows = r;
  p.queries = qv;
  p.n = n;
  p.nq = nq;
  p.nq_pad = nq_pad;
  p.qblocks = (int)(nq_pad / QH);
  p.tiles = (int)((n + HM_HT - 1) / HM_HT);
  p.k = k;
  p.id_offset = id_offset;
  p.err = dev.err;
  p.wait_ns = WAIT_LIMIT_NS;
  p.gfloor = sc.alloc<unsigned long long>((size_t)nq_pad);
  CK(cudaMemsetAsync(p.gfloor, 0, (size_t)nq_pad * 8, s));
  const HammingOut out{out_keys, ids, dist};
  switch (V) {
    case 1: return launch_hamming_v<1>(p, QH, dev, sc, out, s);
    case 2: return launch_hamming_v<2>(p, QH, dev, sc, out, s);
    case 4: return launch_hamming_v<4>(p, QH, dev, sc, out, s);
    case 8: return launch_hamming_v<8>(p, QH, dev, sc, out, s);
    case 16: return launch_hamming_v<16>(p, QH, dev, sc, out, s);
    default: return launch_hamming_v<32>(p, QH, dev, sc, out, s);
  }
}

}  // namespace

void brute_force_knn(const float* base, int64_t n, const float* queries, int64_t nq, int d, int k,
                     Metric metric, int32_t* ids, float* dist, cudaStream_t s,
                     const KnnOptions& options) {
  (void)options;
  require(ids != nullptr || nq == 0, "[mlxvs::brute_force_knn] ids must not be NULL.");
  knn_core(base, n, queries, nq, d, k, metric, 0, nullptr, ids, dist, s);
}

void knn_keys(const float* base, int64_t n, const float* queries, int64_t nq, int d, int k,
              Metric metric, int64_t id_offset, uint64_t* keys, cudaStream_t s) {
  require(keys != nullptr || nq == 0, "[mlxvs::brute_force_knn] keys must not be NULL.");
  knn_core(base, n, queries, nq, d, k, metric, id_offset, keys, nullptr, nullptr, s);
}

void all_neighbors(const float* rows, int64_t n, int d, int k, Metric metric,
                   int64_t query_begin, int64_t query_end, int32_t* ids, float* dist,
                   cudaStream_t s) {
  require(k >= 1 && k <= 255 && n >= 2 && d >= 1,
          "[mlxvs::all_neighbors] 1 <= k <= 255, n >= 2 and d >= 1");
  require(query_begin >= 0 && query_begin <= query_end && query_end <= n,
          "[mlxvs::all_neighbors] 0 <= query_begin <= query_end <= n");
  require(ids != nullptr || query_end == query_begin,
          "[mlxvs::all_neighbors] ids must not be NULL.");
  // every row is a query against all rows, its own row excluded in the
  // kernel (the reference searches k + 1 and drops it in merge_lists)
  knn_core(rows, n, rows + query_begin * d, query_end - query_begin, d, k, metric, 0, nullptr,
           ids, dist, s, query_begin);
}

void topk_merge(const float* scores, int64_t nq, int t, const int32_t* ids, const float* best,
                int id_offset, bool first, int k, int32_t* out_ids, float* out_scores,
                cudaStream_t s) {
  require(k >= 1 && k <= TOPK_KMAX, "[mlxvs::topk_merge] k must be in [1, 256]");
  require(nq >= 0 && t >= 0, "[mlxvs::topk_merge] scores must be float32 [nq, t]");
  if (nq == 0) return;
  require(scores != nullptr || t == 0, "[mlxvs::topk_merge] scores must not be NULL.");
  require(first || (ids != nullptr && best != nullptr),
          "[mlxvs::topk_merge] ids and best [nq, k] are needed unless first.");
  require(out_ids != nullptr && out_scores != nullptr,
          "[mlxvs::topk_merge] outputs must not be NULL.");
  require(nq < (1LL << 31), "[mlxvs::topk_merge] at most 2^31 - 1 rows.");
  device_info();
  TopkRowsParams p{scores, nq, t, first ? nullptr : ids, first ? nullptr : best,
                   id_offset, k, out_ids, out_scores};
  ProfScope prof("topk_rows", s);
  topk_rows_kernel<<<(unsigned)nq, TOPK_THREADS, 0, s>>>(p);
  CK(cudaGetLastError());
}

void refine(const float* dataset, int64_t n, int d, const float* queries, int64_t nq,
            const int32_t* candidates, int c, int k, Metric metric, int32_t* ids, float* dist,
            cudaStream_t s) {
  require(d >= 1 && n >= 0 && nq >= 0 && c >= 0,
          "[mlxvs::refine] dataset [n, d], queries [nq, d] and candidates [nq, c] must match.");
  require(k >= 1 && k <= c, "[mlxvs::refine] k must be in [1, candidates per query].");
  require(k <= TOPK_KMAX, "[mlxvs::refine] k must be at most 256.");
  const int mi = static_cast<int>(metric);
  require(mi >= 0 && mi <= 2, "[mlxvs::refine] unknown metric.");
  require(nq < (1LL << 31), "[mlxvs::refine] at most 2^31 - 1 queries.");
  if (nq == 0) return;
  require(queries != nullptr && candidates != nullptr && ids != nullptr,
          "[mlxvs::refine] null input.");
  require(dataset != nullptr || n == 0, "[mlxvs::refine] null dataset.");
  device_info();
  Scratch sc(s);
  float* sc_scores = sc.alloc<float>((size_t)nq * c);
  float* sel_scores = dist ? dist : sc.alloc<float>((size_t)nq * k);
  RefineParams rp{dataset, n, d, queries, nq, candidates, c, mi, sc_scores};
  {
    const int64_t pairs = nq * (int64_t)c;
    const int warps_per_block = 8;
    const int64_t per_block = (int64_t)warps_per_block * REFINE_ROWS;
    require(pairs / per_block < (1LL << 31), "[mlxvs::refine] too many candidates.");
    ProfScope prof("refine_scores", s);
    refine_scores_kernel<<<(unsigned)((pairs + per_block - 1) / per_block),
                           warps_per_block * 32, 0, s>>>(rp);
    CK(cudaGetLastError());
  }
  // positions 0 .. c-1 as ids: equal scores keep the candidates' order
  TopkRowsParams tp{sc_scores, nq, c, nullptr, nullptr, 0, k, ids, sel_scores};
  {
    ProfScope prof("topk_rows", s);
    topk_rows_kernel<<<(unsigned)nq, TOPK_THREADS, 0, s>>>(tp);
    CK(cudaGetLastError());
  }
  const int64_t count = nq * (int64_t)k;
  ProfScope prof("refine_finish", s);
  refine_finish_kernel<<<(unsigned)((count + 255) / 256), 256, 0, s>>>(
      candidates, c, count, k, metric == Metric::L2 ? 1 : 0, ids, sel_scores);
  CK(cudaGetLastError());
}

void hamming_knn(const uint8_t* rows, int64_t n, const uint8_t* queries, int64_t nq, int bytes,
                 int k, int32_t* ids, float* dist, cudaStream_t s) {
  require(ids != nullptr || nq == 0, "[mlxvs::hamming_knn] ids must not be NULL.");
  hamming_core(rows, n, queries, nq, bytes, k, 0, nullptr, ids, dist, s);
}

void hamming_keys(const uint8_t* rows, int64_t n, const uint8_t* queries, int64_t nq, int bytes,
                  int k, int64_t id_offset, uint64_t* keys, cudaStream_t s) {
  require(keys != nullptr || nq == 0, "[mlxvs::hamming_knn] keys must not be NULL.");
  hamming_core(rows, n, queries, nq, bytes, k, id_offset, keys, nullptr, nullptr, s);
}

void merge_keys(const uint64_t* lists, int num_lists, int64_t nq, int k, int kind,
                const float* queries, int d, int32_t* ids, float* dist, cudaStream_t s) {
  require(k >= 1 && k <= 256, "[mlxvs::merge_keys] k must be in [1, 256].");
  require(num_lists >= 0, "[mlxvs::merge_keys] num_lists must be >= 0.");
  require(nq >= 0 && nq < (1LL << 31), "[mlxvs::merge_keys] nq must be in [0, 2^31).");
  require(kind >= 0 && kind <= KIND_HAMMING, "[mlxvs::merge_keys] unknown kind.");
  require(ids != nullptr || nq == 0, "[mlxvs::merge_keys] ids must not be NULL.");
  DeviceInfo& dev = device_info();
  if (nq == 0) return;
  require(lists != nullptr || num_lists == 0, "[mlxvs::merge_keys] lists must not be NULL.");
  Scratch sc(s);
  float* qq = nullptr;
  // the four-lanes merge computes |q|^2 itself; the others read it from qq
  const bool quad = merge_quad_fits(num_lists, k);
  if (kind == static_cast<int>(Metric::L2)) {
    require(queries != nullptr && d >= 1,
            "[mlxvs::merge_keys] L2 distances need the queries [nq, d].");
  }
  if (kind == static_cast<int>(Metric::L2) && !quad) {
    qq = sc.alloc<float>((size_t)nq);
    unsigned blocks = (unsigned)std::min<int64_t>((nq + 7) / 8, (int64_t)dev.sms * 16);
    ProfScope prof("sumsq", s);
    row_sumsq_kernel<<<blocks, 256, 0, s>>>(queries, nq, d, qq);
    CK(cudaGetLastError());
  }
  if (num_lists == 0) {
    launch_fill(nq * k, kind, ids, dist, nullptr, s);
    return;
  }
  launch_merge(lists, num_lists, nq, nq, k, kind, qq, nullptr, ids, dist, s, 1.0f,
               quad ? queries : nullptr, d);
}

void device_synchronize(cudaStream_t s) {
  DeviceInfo& dev = device_info();
  CK(cudaStreamSynchronize(s));
  uint32_t err = 0;
  CK(cudaMemcpy(&err, dev.err, 4, cudaMemcpyDeviceToHost));
  if (err != 0) {
    CK(cudaMemset(dev.err, 0, 4));
    throw std::runtime_error("[mlxvs_b200] a kernel gave up waiting (error word " +
                             std::to_string(err) + ")");
  }
}

void profile_enable(bool on) {
  std::lock_guard<std::mutex> g(prof_mu);
  for (auto& r : prof_records) {
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  prof_records.clear();
  prof_on = on;
}

void profile_issued(const char* name, double* ops) {
  std::lock_guard<std::mutex> g(prof_mu);
  double total = 0.0;
  for (auto& r : prof_records)
    if (!name || std::strcmp(name, r.name) == 0) total += r.issued;
  if (ops) *ops = total;
}

void profile_read(const char* name, double* total_ms, int64_t* launches) {
  std::lock_guard<std::mutex> g(prof_mu);
  double ms = 0.0;
  int64_t count = 0;
  for (auto& r : prof_records) {
    if (name && std::strcmp(name, r.name) != 0) continue;
    CK(cudaEventSynchronize(r.stop));
    float t = 0.0f;
    CK(cudaEventElapsedTime(&t, r.start, r.stop));
    ms += t;
    ++count;
  }
  if (total_ms) *total_ms = ms;
  if (launches) *launches = count;
}

// ------------------------------------------------------------ peer exchange
// Buffer of one GPU: [flag: u32][failed: u32][pad to 256 B][slot 0 keys]
// [slot 1 keys], from cudaMalloc (IPC handles need it).  The flag holds the
// latest epoch whose keys are complete; failed, the epoch of a step whose
// wait gave up.

constexpr size_t EXCHANGE_HEADER = 256;
// Ample for ranks that reach the merge within one step of each other: the
// time limit guards against a rank that never comes, not against load
// imbalance.
constexpr uint64_t EXCHANGE_WAIT_NS = 30ull * 1000 * 1000 * 1000;

struct Exchange {
  int device = -1;
  int world = 0;
  int rank = 0;
  int64_t capacity = 0;
  uint8_t* own = nullptr;
  uint8_t* peer[MERGE_MAX_PEERS] = {};
  bool opened[MERGE_MAX_PEERS] = {};
};

namespace {
uint64_t* slot_of(uint8_t* buf, int64_t capacity, uint32_t epoch) {
  return reinterpret_cast<uint64_t*>(buf + EXCHANGE_HEADER) + (size_t)(epoch & 1u) * capacity;
}
}  // namespace

Exchange* exchange_create(int world, int rank, int64_t capacity_keys) {
  require(world >= 1 && world <= MERGE_MAX_PEERS,
          "[mlxvs::exchange] world must be in [1, " + std::to_string(MERGE_MAX_PEERS) + "].");
  require(rank >= 0 && rank < world, "[mlxvs::exchange] rank must be in [0, world).");
  require(capacity_keys >= 1, "[mlxvs::exchange] capacity must be at least 1 key.");
  device_info();
  auto x = std::make_unique<Exchange>();
  CK(cudaGetDevice(&x->device));
  x->world = world;
  x->rank = rank;
  x->capacity = capacity_keys;
  const size_t bytes = EXCHANGE_HEADER + 2 * (size_t)capacity_keys * sizeof(uint64_t);
  CK(cudaMalloc(&x->own, bytes));
  CK(cudaMemset(x->own, 0, bytes));
  x->peer[rank] = x->own;
  x->opened[rank] = true;
  return x.release();
}

void exchange_handle(Exchange* x, void* handle) {
  require(x != nullptr && handle != nullptr, "[mlxvs::exchange] null argument.");
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, x->own));
  std::memcpy(handle, &h, sizeof(h));
}

void exchange_open(Exchange* x, int peer, const void* handle) {
  require(x != nullptr && handle != nullptr, "[mlxvs::exchange] null argument.");
  require(peer >= 0 && peer < x->world, "[mlxvs::exchange] peer must be in [0, world).");
  if (peer == x->rank || x->opened[peer]) return;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  x->peer[peer] = static_cast<uint8_t*>(p);
  x->opened[peer] = true;
}

uint64_t* exchange_keys(Exchange* x, uint32_t epoch) {
  require(x != nullptr, "[mlxvs::exchange] null exchange.");
  require(epoch >= 1, "[mlxvs::exchange] epochs start at 1.");
  return slot_of(x->own, x->capacity, epoch);
}

void exchange_merge(Exchange* x, uint32_t epoch, int64_t nq, int k, int kind,
                    const float* queries, int d, int32_t* ids, float* dist, cudaStream_t s) {
  require(x != nullptr, "[mlxvs::exchange] null exchange.");
  require(epoch >= 1, "[mlxvs::exchange] epochs start at 1.");
  require(k >= 1 && merge_quad_fits(x->world, k),
          "[mlxvs::exchange] k must be in [1, 32] with world * k <= " +
              std::to_string(MERGE_QUAD_MAX) + ".");
  require(nq >= 0 && nq * k <= x->capacity, "[mlxvs::exchange] nq * k exceeds the capacity.");
  require(kind >= 0 && kind <= KIND_HAMMING, "[mlxvs::exchange] unknown kind.");
  require(ids != nullptr || nq == 0, "[mlxvs::exchange] ids must not be NULL.");
  require(kind != static_cast<int>(Metric::L2) || nq == 0 || (queries != nullptr && d >= 1),
          "[mlxvs::exchange] L2 distances need the queries [nq, d].");
  for (int r = 0; r < x->world; ++r)
    require(x->opened[r], "[mlxvs::exchange] peer " + std::to_string(r) + " is not opened.");
  int cur = -1;
  CK(cudaGetDevice(&cur));
  require(cur == x->device, "[mlxvs::exchange] the current device is not the exchange's.");
  DeviceInfo& dev = device_info();
  // every step publishes and waits, also with no queries, so that the GPUs'
  // epochs stay in step
  ExchangeFlags f{};
  f.own = reinterpret_cast<volatile uint32_t*>(x->own);
  for (int r = 0; r < x->world; ++r) f.flag[r] = reinterpret_cast<volatile uint32_t*>(x->peer[r]);
  f.world = x->world;
  f.epoch = epoch;
  f.failed = reinterpret_cast<uint32_t*>(x->own) + 1;
  f.err = dev.err;
  f.limit_cycles = (long long)(2 * EXCHANGE_WAIT_NS);
  {
    ProfScope prof("exchange_wait", s);
    exchange_wait_kernel<<<1, 32, 0, s>>>(f);
    CK(cudaGetLastError());
  }
  if (nq == 0) return;
  PeerLists pl{};
  for (int r = 0; r < x->world; ++r) pl.p[r] = slot_of(x->peer[r], x->capacity, epoch);
  pl.failed = f.failed;
  pl.epoch = epoch;
  ProfScope prof("merge", s);
  const unsigned blocks = (unsigned)((nq + 7) / 8);
  const size_t smem = (size_t)x->world * k * 8 * sizeof(uint64_t);
  const float* qrows = kind == static_cast<int>(Metric::L2) ? queries : nullptr;
#define MLXVS_MERGE_PEERS(KR_)                                                           \
  merge_keys_quad_kernel<KR_, true><<<blocks, 32, smem, s>>>(                          \
      nullptr, x->world, nq, nq, k, kind, nullptr, nullptr, ids, dist, 1.0f, qrows, d, pl)
  if (k <= 10)
    MLXVS_MERGE_PEERS(10);
  else if (k <= 16)
    MLXVS_MERGE_PEERS(16);
  else
    MLXVS_MERGE_PEERS(32);
#undef MLXVS_MERGE_PEERS
  CK(cudaGetLastError());
}

void exchange_destroy(Exchange* x) {
  if (x == nullptr) return;
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != x->device) cudaSetDevice(x->device);
  cudaDeviceSynchronize();
  for (int r = 0; r < x->world; ++r)
    if (r != x->rank && x->opened[r] && x->peer[r]) cudaIpcCloseMemHandle(x->peer[r]);
  cudaFree(x->own);
  if (cur >= 0 && cur != x->device) cudaSetDevice(cur);
  delete x;
}

const char* version() { return MLXVS_B200_VERSION; }

}  // namespace mlxvs_b200

// ------------------------------------------------------ no-allocation entry
// Hamming k-NN for callers that must not allocate device memory.  Its
// scratch (the units' partial lists, the shared floors and an error word)
// is the file-scope array below, which every GPU that loads this library
// holds until the process exits; no call here allocates or frees.
namespace mlxvs_b200 {

namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(16) << 20;  // 16 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

struct NoAllocDevice {
  unsigned char* scratch = nullptr;  // device address of g_noalloc_scratch
  int sms = 0;
  int max_smem = 0;
};

// Set-up, once per device with that device current: the array's device
// address (host code cannot use the symbol itself) and the device limits.
const NoAllocDevice& noalloc_device() {
  static std::mutex mu;
  static NoAllocDevice devs[64];
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64)
    throw std::runtime_error("[mlxvs_b200] device ordinal " + std::to_string(dev) +
                             " is beyond the 64 devices this library tracks");
  std::lock_guard<std::mutex> guard(mu);
  NoAllocDevice& d = devs[dev];
  if (d.scratch == nullptr) {
    int major = 0, minor = 0;
    CK(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    CK(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (major != 10 || minor != 0)
      throw std::runtime_error("[mlxvs_b200] needs an sm_100 GPU (B200); device " +
                               std::to_string(dev) + " is sm_" + std::to_string(major) +
                               std::to_string(minor));
    CK(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    CK(cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      throw std::runtime_error(std::string("[mlxvs_b200] cudaGetSymbolAddress failed: ") +
                               cudaGetErrorString(e));
    }
    d.scratch = static_cast<unsigned char*>(p);
  }
  return d;
}

template <int V, int QH>
void noalloc_hamming_launch(HammingParams p, const NoAllocDevice& dev, size_t list_room,
                            int32_t* ids, float* dist, cudaStream_t s) {
  auto kern = hamming_topk_kernel<V, QH>;
  int stages = 4;
  uint32_t smem = hamming_smem_bytes(V, QH, p.k, stages);
  while (smem > (uint32_t)dev.max_smem && stages > 2)
    smem = hamming_smem_bytes(V, QH, p.k, --stages);
  if (smem > (uint32_t)dev.max_smem)
    throw std::runtime_error("[mlxvs_b200] hamming: no kernel shape fits shared memory");
  p.stages = stages;
  CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 1;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, QH + 32, smem));
  const int slots = dev.sms * std::max(per_sm, 1);
  // as many base ranges per query block as the scratch holds lists for
  const size_t per_split = (size_t)p.nq_pad * p.k * 8;
  const int fit = (int)std::min<size_t>(64, list_room / per_split);
  p.splits = std::min(choose_splits(p.qblocks, p.tiles, slots, 2.0, 64), fit);
  p.units = p.qblocks * p.splits;
  {
    ProfScope prof("hamming_topk", s);
    kern<<<std::min(p.units, slots), QH + 32, smem, s>>>(p);
    CK(cudaGetLastError());
  }
  launch_merge(p.partial, p.splits, p.nq_pad, p.nq, p.k, KIND_HAMMING, nullptr, nullptr, ids,
               dist, s);
}

}  // namespace

void hamming_knn_noalloc(const uint8_t* rows, int64_t n, const uint8_t* queries, int64_t nq,
                         int bytes, int k, int32_t* ids, float* dist, cudaStream_t s) {
  const char* op = "[mlxvs::hamming_knn_noalloc] ";
  require(ids != nullptr || nq == 0, std::string(op) + "ids must not be NULL.");
  require(k >= 1 && k <= 256, std::string(op) + "k must be in [1, 256].");
  require(n >= 0 && n < (1LL << 31), std::string(op) + "the number of rows must be in [0, 2^31).");
  require(nq >= 0 && nq < (1LL << 31),
          std::string(op) + "the number of queries must be in [0, 2^31).");
  int V = 0;
  for (int v = 1; v <= 32; v <<= 1)
    if (16 * v == bytes) V = v;
  require(V != 0, std::string(op) +
                      "bytes must be 16, 32, 64, 128, 256 or 512: the codes are read in place "
                      "(a padded copy would need an allocation).");
  require((rows == nullptr || (reinterpret_cast<uintptr_t>(rows) & 15) == 0) &&
              (queries == nullptr || (reinterpret_cast<uintptr_t>(queries) & 15) == 0),
          std::string(op) + "rows and queries must be 16-byte aligned.");
  const NoAllocDevice& dev = noalloc_device();
  if (nq == 0) return;
  if (n == 0) {
    launch_fill(nq * k, KIND_HAMMING, ids, dist, nullptr, s);
    return;
  }
  require(rows != nullptr && queries != nullptr, std::string(op) + "null input.");
  int QH = 256;
  while (QH > 64 && (uint32_t)QH * k * 8u > 64u * 1024u) QH >>= 1;
  if (V > 16 && QH > 128) QH = 128;
  const int64_t nq_pad = round_up(nq, QH);
  // scratch layout: error word | shared floors [nq_pad] | lists [splits][nq_pad][k]
  const size_t floors_off = 256;
  const size_t lists_off = (size_t)round_up(floors_off + (size_t)nq_pad * 8, 256);
  const size_t one_split = (size_t)nq_pad * k * 8;
  if (lists_off + one_split > NOALLOC_SCRATCH_BYTES)
    throw std::invalid_argument(
        std::string(op) + "nq * k is too large for the 16 MiB static scratch: it needs " +
        std::to_string(lists_off + one_split) + " bytes (at most about 2^21 / (k + 1) queries).");
  HammingParams p{};
  p.rows = rows;
  p.queries = queries;
  p.n = n;
  p.nq = nq;
  p.nq_pad = nq_pad;
  p.qblocks = (int)(nq_pad / QH);
  p.tiles = (int)((n + HM_HT - 1) / HM_HT);
  p.k = k;
  p.id_offset = 0;
  p.err = reinterpret_cast<uint32_t*>(dev.scratch);
  p.wait_ns = WAIT_LIMIT_NS;
  p.gfloor = reinterpret_cast<unsigned long long*>(dev.scratch + floors_off);
  p.partial = reinterpret_cast<uint64_t*>(dev.scratch + lists_off);
  // the array keeps the previous call's contents: clear the error word and
  // the floors, which must start at zero (every list slot is rewritten)
  CK(cudaMemsetAsync(dev.scratch, 0, lists_off, s));
  const size_t room = NOALLOC_SCRATCH_BYTES - lists_off;
  switch (V) {
#define MLXVS_NOALLOC_V(V_)                                                   \
  case V_:                                                                    \
    if (QH == 256) noalloc_hamming_launch<V_, 256>(p, dev, room, ids, dist, s); \
    else if (QH == 128) noalloc_hamming_launch<V_, 128>(p, dev, room, ids, dist, s); \
    else noalloc_hamming_launch<V_, 64>(p, dev, room, ids, dist, s);        \
    break;
    MLXVS_NOALLOC_V(1)
    MLXVS_NOALLOC_V(2)
    MLXVS_NOALLOC_V(4)
#undef MLXVS_NOALLOC_V
    case 8:
      if (QH == 256) noalloc_hamming_launch<8, 256>(p, dev, room, ids, dist, s);
      else if (QH == 128) noalloc_hamming_launch<8, 128>(p, dev, room, ids, dist, s);
      else noalloc_hamming_launch<8, 64>(p, dev, room, ids, dist, s);
      break;
    case 16:
      if (QH == 256) noalloc_hamming_launch<16, 256>(p, dev, room, ids, dist, s);
      else if (QH == 128) noalloc_hamming_launch<16, 128>(p, dev, room, ids, dist, s);
      else noalloc_hamming_launch<16, 64>(p, dev, room, ids, dist, s);
      break;
    default:
      if (QH == 128) noalloc_hamming_launch<32, 128>(p, dev, room, ids, dist, s);
      else noalloc_hamming_launch<32, 64>(p, dev, room, ids, dist, s);
      break;
  }
  // report a kernel that gave up waiting: the call returns after its work
  uint32_t err = 0;
  CK(cudaMemcpyAsync(&err, dev.scratch, 4, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  if (err != 0)
    throw std::runtime_error("[mlxvs_b200] a kernel gave up waiting (error word " +
                             std::to_string(err) + ")");
}

}  // namespace mlxvs_b200
