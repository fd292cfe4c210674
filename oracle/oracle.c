/*
 * CPU oracle for mlxVS's exact k-NN hot path.  TEST INFRASTRUCTURE ONLY:
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it as
 * the checker / CPU baseline; the product library never calls it.
 *
 * Restates, in plain C with OpenMP:
 *   brute_force_knn  src/knn.cpp:71-142
 *   unit_rows        src/knn.cpp:30-33            (cosine)
 *   float_rows       src/utils.h:18-29            (caller casts to float32)
 *   topk_merge       src/knn.cpp:37-69, src/kernels.h:14-229 (order, padding)
 *   hamming_knn      src/ivf.cpp:1343-1403, pack_words :1123-1135,
 *                    IVF_BINARY_SCAN_SOURCE src/ivf_kernels.h:577-594
 *
 * Parity is pinned by the reference's known-answer tests (see oracle.h); the
 * reference itself cannot run here (MLX + Metal).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* src/kernels.h:16-19: a float as an unsigned int that sorts the same way. */
static inline uint32_t order_bits(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static inline float from_order_bits(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k ^ 0x80000000u) : ~k;
  float v;
  memcpy(&v, &u, 4);
  return v;
}

uint64_t oracle_key(float score, int32_t id) {
  return ((uint64_t)order_bits(score) << 32) | (uint64_t)(uint32_t)(~(uint32_t)id);
}

static inline int32_t key_id(uint64_t key) {
  return key == 0 ? -1 : (int32_t)(~(uint32_t)(key & 0xffffffffu));
}

static inline float key_score(uint64_t key) {
  return key == 0 ? -INFINITY : from_order_bits((uint32_t)(key >> 32));
}

/* Min-heap of the k best keys seen (root = the worst kept); 0 = empty. */
static inline void heap_push(uint64_t* h, int k, uint64_t key) {
  if (key <= h[0]) return;
  int i = 0;
  for (;;) {
    int l = 2 * i + 1, r = l + 1, m = i;
    uint64_t mv = key;
    if (l < k && h[l] < mv) { m = l; mv = h[l]; }
    if (r < k && h[r] < mv) { m = r; mv = h[r]; }
    if (m == i) break;
    h[i] = h[m];
    i = m;
  }
  h[i] = key;
}

static int cmp_desc(const void* a, const void* b) {
  uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
  return x < y ? 1 : (x > y ? -1 : 0);
}

/* unit_rows (src/knn.cpp:30-33): x / max(sqrt(sum x^2), 1e-30), float32. */
static float* unit_rows(const float* x, int64_t n, int32_t d) {
  float* y = (float*)malloc((size_t)(n > 0 ? n : 1) * (size_t)d * sizeof(float));
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float* r = x + (size_t)i * d;
    float ss = 0.0f;
    for (int32_t t = 0; t < d; ++t) ss += r[t] * r[t];
    float norm = sqrtf(ss);
    float den = norm > 1e-30f ? norm : 1e-30f;
    for (int32_t t = 0; t < d; ++t) y[(size_t)i * d + t] = r[t] / den;
  }
  return y;
}

enum { QBLK = 16, RBLK = 512 };

/* The best k keys of every query, best first, into keys [nq][k]. */
static void knn_core(const float* base, int64_t n, const float* queries,
                     int64_t nq, int32_t d, int32_t k, int32_t metric,
                     int64_t id_offset, uint64_t* keys) {
  const float* b = base;
  const float* q = queries;
  float* bu = NULL;
  float* qu = NULL;
  if (metric == ORACLE_COSINE) {
    bu = unit_rows(base, n, d);
    qu = unit_rows(queries, nq, d);
    b = bu;
    q = qu;
  }
  /* |b|^2 per base row for L2 (src/knn.cpp:115) */
  float* nb = (float*)calloc((size_t)(n > 0 ? n : 1), sizeof(float));
  if (metric == ORACLE_L2) {
#pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < n; ++j) {
      const float* r = b + (size_t)j * d;
      float ss = 0.0f;
      for (int32_t t = 0; t < d; ++t) ss += r[t] * r[t];
      nb[j] = ss;
    }
  }
  /* tasks: (block of QBLK queries, chunk of base rows), enough of them to
     keep every thread busy also when there are few queries; each task keeps
     its own heaps, merged per query at the end */
  int64_t blocks = (nq + QBLK - 1) / QBLK;
  int64_t chunks = 1;
#ifdef _OPENMP
  {
    int64_t want = 4 * (int64_t)omp_get_max_threads();
    chunks = (want + blocks - 1) / (blocks > 0 ? blocks : 1);
    int64_t max_chunks = (n + RBLK - 1) / RBLK;
    if (chunks > max_chunks) chunks = max_chunks;
    if (chunks < 1) chunks = 1;
  }
#endif
  const int64_t rows_per_chunk = ((n + chunks - 1) / chunks + RBLK - 1) / RBLK * RBLK;
  uint64_t* task_heaps =
      (uint64_t*)calloc((size_t)(blocks > 0 ? blocks : 1) * chunks * QBLK * k, sizeof(uint64_t));
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t task = 0; task < blocks * chunks; ++task) {
    int64_t blk = task / chunks, ch = task % chunks;
    int64_t i0 = blk * QBLK;
    int64_t i1 = i0 + QBLK < nq ? i0 + QBLK : nq;
    int64_t r0 = ch * rows_per_chunk;
    int64_t r1 = r0 + rows_per_chunk < n ? r0 + rows_per_chunk : n;
    uint64_t* heaps = task_heaps + (size_t)task * QBLK * k;
    for (int64_t j0 = r0; j0 < r1; j0 += RBLK) {
      int64_t j1 = j0 + RBLK < r1 ? j0 + RBLK : r1;
      for (int64_t i = i0; i < i1; ++i) {
        const float* qi = q + (size_t)i * d;
        uint64_t* h = heaps + (size_t)(i - i0) * k;
        for (int64_t j = j0; j < j1; ++j) {
          const float* bj = b + (size_t)j * d;
          float dot = 0.0f;
#pragma omp simd reduction(+ : dot)
          for (int32_t t = 0; t < d; ++t) dot += qi[t] * bj[t];
          float s = dot;
          if (metric == ORACLE_L2) {
            /* 2 q.b - |b|^2 (src/knn.cpp:111-116) */
            float two = 2.0f * dot;
            s = two - nb[j];
          }
          uint64_t key = oracle_key(s, (int32_t)(j + id_offset));
          if (key > h[0]) heap_push(h, k, key);
        }
      }
    }
  }
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < nq; ++i) {
    int64_t blk = i / QBLK;
    uint64_t* h = (uint64_t*)calloc((size_t)k, sizeof(uint64_t));
    for (int64_t ch = 0; ch < chunks; ++ch) {
      const uint64_t* src = task_heaps + ((size_t)(blk * chunks + ch) * QBLK + (i - blk * QBLK)) * k;
      for (int32_t j = 0; j < k; ++j)
        if (src[j] > h[0]) heap_push(h, k, src[j]);
    }
    qsort(h, (size_t)k, sizeof(uint64_t), cmp_desc);
    memcpy(keys + (size_t)i * k, h, (size_t)k * sizeof(uint64_t));
    free(h);
  }
  free(task_heaps);
  free(nb);
  free(bu);
  free(qu);
}

static int set_threads(int32_t threads) {
#ifdef _OPENMP
  int old = omp_get_max_threads();
  if (threads > 0) omp_set_num_threads(threads);
  return old;
#else
  (void)threads;
  return 1;
#endif
}

static void restore_threads(int old) {
#ifdef _OPENMP
  omp_set_num_threads(old);
#else
  (void)old;
#endif
}

int oracle_knn_keys(const float* base, int64_t n, const float* queries,
                    int64_t nq, int32_t d, int32_t k, int32_t metric,
                    int64_t id_offset, uint64_t* keys, int32_t threads) {
  if (k < 1 || k > 256 || d < 1 || n < 0 || nq < 0) return 1;
  if (metric < 0 || metric > 2) return 1;
  int old = set_threads(threads);
  knn_core(base, n, queries, nq, d, k, metric, id_offset, keys);
  restore_threads(old);
  return 0;
}

int oracle_brute_force_knn(const float* base, int64_t n, const float* queries,
                           int64_t nq, int32_t d, int32_t k, int32_t metric,
                           int32_t* ids, float* distances, int32_t threads) {
  if (k < 1 || k > 256 || d < 1 || n < 0 || nq < 0) return 1;
  if (metric < 0 || metric > 2) return 1;
  int old = set_threads(threads);
  uint64_t* keys = (uint64_t*)malloc((size_t)(nq > 0 ? nq : 1) * (size_t)k * sizeof(uint64_t));
  knn_core(base, n, queries, nq, d, k, metric, 0, keys);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < nq; ++i) {
    float qq = 0.0f;
    if (metric == ORACLE_L2) {
      const float* qi = queries + (size_t)i * d;
      for (int32_t t = 0; t < d; ++t) qq += qi[t] * qi[t];
    }
    for (int32_t j = 0; j < k; ++j) {
      uint64_t key = keys[(size_t)i * k + j];
      int32_t id = key_id(key);
      float best = key_score(key);
      ids[(size_t)i * k + j] = id;
      if (distances) {
        if (metric == ORACLE_L2) {
          /* src/knn.cpp:122-131: max(|q|^2 - best, 0), +inf where missing */
          float dd = qq - best;
          distances[(size_t)i * k + j] = id >= 0 ? (dd > 0.0f ? dd : 0.0f) : INFINITY;
        } else {
          distances[(size_t)i * k + j] = best; /* -inf where missing */
        }
      }
    }
  }
  free(keys);
  restore_threads(old);
  return 0;
}

static inline int popcount_bytes(const uint8_t* a, const uint8_t* b, int32_t bytes) {
  int h = 0;
  int32_t t = 0;
  for (; t + 8 <= bytes; t += 8) {
    uint64_t x, y;
    memcpy(&x, a + t, 8);
    memcpy(&y, b + t, 8);
    h += __builtin_popcountll(x ^ y);
  }
  for (; t < bytes; ++t) h += __builtin_popcount((unsigned)(a[t] ^ b[t]));
  return h;
}

int oracle_hamming_knn(const uint8_t* rows, int64_t n, const uint8_t* queries,
                       int64_t nq, int32_t bytes, int32_t k, int32_t* ids,
                       float* distances, int32_t threads) {
  if (k < 1 || k > 256 || bytes < 1 || n < 0 || nq < 0) return 1;
  int old = set_threads(threads);
  int64_t blocks = (nq + QBLK - 1) / QBLK;
  int64_t chunks = 1;
#ifdef _OPENMP
  {
    int64_t want = 4 * (int64_t)omp_get_max_threads();
    chunks = (want + blocks - 1) / (blocks > 0 ? blocks : 1);
    int64_t max_chunks = (n + RBLK - 1) / RBLK;
    if (chunks > max_chunks) chunks = max_chunks;
    if (chunks < 1) chunks = 1;
  }
#endif
  const int64_t rows_per_chunk = ((n + chunks - 1) / chunks + RBLK - 1) / RBLK * RBLK;
  uint64_t* task_heaps =
      (uint64_t*)calloc((size_t)(blocks > 0 ? blocks : 1) * chunks * QBLK * k, sizeof(uint64_t));
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t task = 0; task < blocks * chunks; ++task) {
    int64_t blk = task / chunks, ch = task % chunks;
    int64_t i0 = blk * QBLK;
    int64_t i1 = i0 + QBLK < nq ? i0 + QBLK : nq;
    int64_t r0 = ch * rows_per_chunk;
    int64_t r1 = r0 + rows_per_chunk < n ? r0 + rows_per_chunk : n;
    uint64_t* heaps = task_heaps + (size_t)task * QBLK * k;
    for (int64_t j0 = r0; j0 < r1; j0 += RBLK) {
      int64_t j1 = j0 + RBLK < r1 ? j0 + RBLK : r1;
      for (int64_t i = i0; i < i1; ++i) {
        const uint8_t* qi = queries + (size_t)i * bytes;
        uint64_t* h = heaps + (size_t)(i - i0) * k;
        for (int64_t j = j0; j < j1; ++j) {
          int hd = popcount_bytes(qi, rows + (size_t)j * bytes, bytes);
          /* nearest first, then lower id: the key of -distance */
          uint64_t key = oracle_key(-(float)hd, (int32_t)j);
          if (key > h[0]) heap_push(h, k, key);
        }
      }
    }
  }
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < nq; ++i) {
    int64_t blk = i / QBLK;
    uint64_t* h = (uint64_t*)calloc((size_t)k, sizeof(uint64_t));
    for (int64_t ch = 0; ch < chunks; ++ch) {
      const uint64_t* src = task_heaps + ((size_t)(blk * chunks + ch) * QBLK + (i - blk * QBLK)) * k;
      for (int32_t j = 0; j < k; ++j)
        if (src[j] > h[0]) heap_push(h, k, src[j]);
    }
    qsort(h, (size_t)k, sizeof(uint64_t), cmp_desc);
    for (int32_t j = 0; j < k; ++j) {
      int32_t id = key_id(h[j]);
      ids[(size_t)i * k + j] = id;
      if (distances)
        distances[(size_t)i * k + j] = id >= 0 ? -key_score(h[j]) : INFINITY;
    }
    free(h);
  }
  free(task_heaps);
  restore_threads(old);
  return 0;
}

/* The best k distinct keys of L lists per query, best first (0 = empty):
 * a key that sits in several lists (the GPU search's units start from an
 * earlier unit's list) is taken once. */
void oracle_merge_keys(const uint64_t* lists, int32_t L, int64_t nq, int32_t k,
                       uint64_t* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < nq; ++i) {
    uint64_t* h = (uint64_t*)calloc((size_t)k, sizeof(uint64_t));
    for (int32_t l = 0; l < L; ++l)
      for (int32_t j = 0; j < k; ++j) {
        uint64_t key = lists[((size_t)l * nq + i) * k + j];
        if (key <= h[0]) continue;
        int held = 0;
        for (int32_t s = 0; s < k && !held; ++s) held = h[s] == key;
        if (!held) heap_push(h, k, key);
      }
    qsort(h, (size_t)k, sizeof(uint64_t), cmp_desc);
    memcpy(out + (size_t)i * k, h, (size_t)k * sizeof(uint64_t));
    free(h);
  }
}
