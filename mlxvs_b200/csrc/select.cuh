// Row-wise selection: the standalone topk_merge (one merge step of the
// reference's tile loop, src/knn.cpp:37-69 with its kernel src/kernels.h:
// 37-229) and the exact re-ranking refine (src/ivf.cpp:1642-1708), which
// scores each query's candidates and selects with the same kernel.
#pragma once

#include "common.cuh"

namespace mlxvs_b200 {

constexpr int TOPK_THREADS = 256;  // threads per row (the reference's TOPK_THREADS)
constexpr int TOPK_KMAX = 256;     // the largest k (TOPK_MAX)

struct TopkRowsParams {
  const float* scores;       // [nq][t] (row stride t)
  int64_t nq;
  int32_t t;
  const int32_t* prev_ids;   // [nq][k] running list, or null (first)
  const float* prev_scores;  // [nq][k]
  int32_t id_offset;         // column j has id id_offset + j
  int32_t k;
  int32_t* out_ids;          // [nq][k]
  float* out_scores;         // [nq][k]
};

// The radix select stops once its bucket holds at most this many entries
// and sorts those instead.
constexpr int TOPK_BUCKET = 256;

// Sorts keys[0 .. n) in shared memory, largest first (a bitonic network
// over the next power of two; the caller has zeroed the slots past n, and
// zero is below every real key).  Every thread of the block calls it.
__device__ __forceinline__ void bitonic_desc_u64(unsigned long long* keys, uint32_t n, int lid) {
  uint32_t size_pow2 = 1;
  while (size_pow2 < n) size_pow2 <<= 1;
  for (uint32_t size = 2; size <= size_pow2; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t i = lid; i < size_pow2; i += TOPK_THREADS) {
        const uint32_t j = i ^ stride;
        if (j > i) {
          const bool forward = (i & size) == 0;
          const unsigned long long a = keys[i], b = keys[j];
          if (forward != (a > b)) {
            keys[i] = b;
            keys[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

// "a comes before b": higher score first, then lower id as unsigned (so -1
// goes last); src/kernels.h:21-23.
__device__ __forceinline__ bool topk_before(float sa, int32_t ia, float sb, int32_t ib) {
  return sa > sb || (sa == sb && (uint32_t)ia < (uint32_t)ib);
}

// One block per row.  Candidates are the row's t scores and, unless first,
// the k running entries; each is the 64-bit key (order bits of the score,
// ~id), larger = better, so one radix select over the keys (8-bit digits
// from the top, stopping as soon as the selected bucket is taken whole)
// finds the k-th largest key and how many entries equal to it to keep.  One
// pass gathers the winners; a bitonic sort orders them by topk_before.
__global__ void __launch_bounds__(TOPK_THREADS) topk_rows_kernel(TopkRowsParams p) {
  constexpr int WARPS = TOPK_THREADS / 32;
  __shared__ uint32_t hist[WARPS][256];
  __shared__ uint32_t suffix[256];
  __shared__ unsigned long long s_prefix;
  __shared__ uint32_t s_need, s_done;
  __shared__ uint32_t taken_above, taken_equal;
  __shared__ float sel_score[TOPK_KMAX];
  __shared__ int32_t sel_id[TOPK_KMAX];
  __shared__ unsigned long long bucket[TOPK_BUCKET];
  __shared__ uint32_t s_count, n_bucket;

  const int lid = threadIdx.x;
  const int warp = lid >> 5;
  const int64_t q = blockIdx.x;
  if (q >= p.nq) return;
  const uint32_t t = (uint32_t)p.t;
  const uint32_t k = (uint32_t)p.k;
  const bool has_prev = p.prev_ids != nullptr;
  const uint32_t total = t + (has_prev ? k : 0u);
  const uint32_t keff = k < total ? k : total;
  const float* row = p.scores + q * (int64_t)t;
  const int64_t prev = q * (int64_t)k;

  auto candidate = [&](uint32_t i, float& v, int32_t& id) {
    if (i < t) {
      v = row[i];
      id = p.id_offset + (int32_t)i;
    } else {
      v = p.prev_scores[prev + (i - t)];
      id = p.prev_ids[prev + (i - t)];
    }
  };
  auto key_of = [](float v, int32_t id) -> uint64_t {
    return ((uint64_t)order_bits(v) << 32) | (uint64_t)(~(uint32_t)id);
  };

  uint64_t prefix = 0, mask = 0;
  uint32_t need = keff;
  bool compact = false;
  if (keff > 0) {
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int i = lid; i < WARPS * 256; i += TOPK_THREADS) (&hist[0][0])[i] = 0u;
      __syncthreads();
      for (uint32_t i = lid; i < total; i += TOPK_THREADS) {
        float v;
        int32_t id;
        candidate(i, v, id);
        const uint64_t key = key_of(v, id);
        if ((key & mask) == prefix) atomicAdd(&hist[warp][(uint32_t)(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      // per digit (one per thread) its count, then the counts of every digit
      // at or above it; the selected digit is where that first reaches need
      uint32_t c = 0;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) c += hist[w][lid];
      suffix[lid] = c;
      __syncthreads();
      for (int off = 1; off < 256; off <<= 1) {
        const uint32_t add = lid + off < 256 ? suffix[lid + off] : 0u;
        __syncthreads();
        suffix[lid] += add;
        __syncthreads();
      }
      const uint32_t at_or_above = suffix[lid];
      const uint32_t above = at_or_above - c;
      if (at_or_above >= need && above < need) {
        s_prefix = prefix | ((uint64_t)lid << shift);
        s_need = need - above;
        s_done = (c == need - above) ? 1u : 0u;
        s_count = c;
      }
      __syncthreads();
      prefix = s_prefix;
      need = s_need;
      mask |= 255ull << shift;
      const bool done = s_done != 0;
      compact = !done && s_count <= (uint32_t)TOPK_BUCKET;
      __syncthreads();
      if (done || compact) break;
    }
  }

  // gather: every key above the k-th, and `need` of those equal to it (equal
  // keys are equal entries, so which of them is immaterial); when the
  // selected bucket is small, its keys instead, whose best `need` a sort in
  // shared memory picks (instead of more passes over the row)
  if (lid == 0) {
    taken_above = 0;
    taken_equal = 0;
    n_bucket = 0;
  }
  for (int i = lid; i < TOPK_KMAX; i += TOPK_THREADS) {
    sel_score[i] = -INFINITY;
    sel_id[i] = -1;
  }
  for (int i = lid; i < TOPK_BUCKET; i += TOPK_THREADS) bucket[i] = 0ull;
  __syncthreads();
  const uint32_t n_above = keff - need;
  if (keff > 0) {
    for (uint32_t i = lid; i < total; i += TOPK_THREADS) {
      float v;
      int32_t id;
      candidate(i, v, id);
      const uint64_t full = key_of(v, id);
      const uint64_t key = full & mask;
      if (key > prefix) {
        const uint32_t at = atomicAdd(&taken_above, 1u);
        sel_score[at] = v;
        sel_id[at] = id;
      } else if (key == prefix) {
        if (compact) {
          bucket[atomicAdd(&n_bucket, 1u)] = full;
        } else {
          const uint32_t at = atomicAdd(&taken_equal, 1u);
          if (at < need) {
            sel_score[n_above + at] = v;
            sel_id[n_above + at] = id;
          }
        }
      }
    }
  }
  __syncthreads();
  if (compact) {
    bitonic_desc_u64(bucket, n_bucket, lid);
    for (uint32_t i = lid; i < need; i += TOPK_THREADS) {
      const uint64_t key = bucket[i];
      sel_score[n_above + i] = from_order_bits((uint32_t)(key >> 32));
      sel_id[n_above + i] = (int32_t)(~(uint32_t)key);
    }
    __syncthreads();
  }

  // bitonic sort of the winners, best first (src/kernels.h:196-222)
  uint32_t size_pow2 = 1;
  while (size_pow2 < keff) size_pow2 <<= 1;
  for (uint32_t size = 2; size <= size_pow2; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t i = lid; i < size_pow2; i += TOPK_THREADS) {
        const uint32_t j = i ^ stride;
        if (j > i) {
          const bool forward = (i & size) == 0;
          const float si = sel_score[i], sj = sel_score[j];
          const int32_t ii = sel_id[i], ij = sel_id[j];
          const bool in_order = topk_before(si, ii, sj, ij);
          if (forward != in_order) {
            sel_score[i] = sj;
            sel_score[j] = si;
            sel_id[i] = ij;
            sel_id[j] = ii;
          }
        }
      }
      __syncthreads();
    }
  }
  for (uint32_t i = lid; i < k; i += TOPK_THREADS) {
    const bool ok = i < keff;
    p.out_scores[prev + i] = ok ? sel_score[i] : -INFINITY;
    p.out_ids[prev + i] = ok ? sel_id[i] : -1;
  }
}

// Large k, between the two passes: each of G disjoint samples of the base
// (split g of the first pass) holds its exact best kg keys for query q, so
// the smallest of their kg-th keys has at least G * kg >= k rows at or above
// it and is a floor of the final k-th best.  floor[q] is that key minus one
// (the key itself must pass), or 0 when some sample list is not full.
__global__ void sample_floor_kernel(const uint64_t* __restrict__ lists, int32_t groups,
                                    int64_t nq_pad, int32_t kg, int64_t nq,
                                    unsigned long long* __restrict__ floor) {
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq_pad) return;
  uint64_t f = ~0ull;
  if (q < nq) {
    for (int g = 0; g < groups; ++g) {
      const uint64_t worst = lists[((size_t)g * nq_pad + q) * kg];  // lists are worst first
      f = worst < f ? worst : f;
    }
  } else {
    f = 0;
  }
  floor[q] = f == 0 ? 0ull : (unsigned long long)(f - 1);
}

// The floor of the listed-sample search: each query's kp-th best key of the
// sample (merged lists, best first), less one; 0 (no floor) when the sample
// held fewer than kp rows or for padding rows.
__global__ void list_floor_kernel(const uint64_t* __restrict__ top, int32_t kp, int64_t nq,
                                  int64_t nq_pad, unsigned long long* __restrict__ floor) {
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq_pad) return;
  const uint64_t f = q < nq ? top[(size_t)q * kp + kp - 1] : 0ull;
  floor[q] = f == 0 ? 0ull : (unsigned long long)(f - 1);
}

// One fp16 pass on inexact operands: lowers each query's floor (a key F - 1,
// from sample_floor_kernel) by 2 eps, eps bounding |fp16 score - exact
// score| in the same units: every row of the exact best k then scores at
// least F - 2 eps in the fp16 pass.  The new floor is the key of that score
// (rounded down) with the lowest id part.
__global__ void margin_floor_kernel(unsigned long long* __restrict__ floor, int64_t nq,
                                    float eps) {
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const uint64_t f = floor[q];
  if (f == 0) return;
  const float s = __fsub_rd(key_score(f + 1), 2.0f * eps);
  floor[q] = (unsigned long long)order_bits(s) << 32;
}

struct RescoreParams {
  const float* base;      // [n][d] float32, the caller's rows
  const float* queries;   // [nq][d]
  int64_t n;
  int32_t d;
  int64_t id_offset;      // ids in the keys are id_offset + row
  int32_t metric;         // 0 inner product, 1 L2, 2 cosine
  uint64_t* cand;         // [splits][nq_pad][cap] keys, rewritten in place
  const int32_t* count;   // [splits][nq_pad]
  int32_t splits;
  int64_t nq;
  int64_t nq_pad;
  int32_t cap;
};

// The kept candidates' keys with exact float32 scores in the reference's
// form (src/knn.cpp:111-116: L2 2 q.b - |b|^2, inner product q.b, cosine
// q.b / (max(|q|, 1e-30) max(|b|, 1e-30))), one warp per (split, query)
// walking its candidates; the row is read from the caller's float32 base.
__global__ void rescore_kernel(RescoreParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t pair = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (pair >= (int64_t)p.splits * p.nq) return;
  const int32_t sp = (int32_t)(pair / p.nq);
  const int64_t q = pair - (int64_t)sp * p.nq;
  int32_t cnt = p.count[(size_t)sp * p.nq_pad + q];
  cnt = cnt < p.cap ? cnt : p.cap;
  if (cnt <= 0) return;
  const float* x = p.queries + q * p.d;
  float qq = 0.0f;
  if (p.metric == 2) {
    for (int j = lane; j < p.d; j += 32) qq = fmaf(x[j], x[j], qq);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) qq += __shfl_xor_sync(0xffffffffu, qq, off);
  }
  uint64_t* keys = p.cand + ((size_t)sp * p.nq_pad + q) * (size_t)p.cap;
  for (int32_t i = 0; i < cnt; ++i) {
    const uint64_t key = keys[i];
    const uint32_t id = ~(uint32_t)key;
    const float* r = p.base + ((int64_t)id - p.id_offset) * p.d;
    float dot = 0.0f, rr = 0.0f;
    for (int j = lane; j < p.d; j += 32) {
      const float a = __ldg(r + j);
      dot = fmaf(a, x[j], dot);
      rr = fmaf(a, a, rr);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      dot += __shfl_xor_sync(0xffffffffu, dot, off);
      rr += __shfl_xor_sync(0xffffffffu, rr, off);
    }
    float sc;
    if (p.metric == 1)
      sc = 2.0f * dot - rr;
    else if (p.metric == 2)
      sc = dot / (fmaxf(sqrtf(qq), 1e-30f) * fmaxf(sqrtf(rr), 1e-30f));
    else
      sc = dot;
    if (lane == 0) keys[i] = make_key(sc, id);
  }
}

// Large k, last step: the best k keys of the candidates the collecting pass
// kept for each query (splits x cap keys, count[s * nq_pad + q] of them per
// split), best first, 0-padded; a count above cap (candidates dropped) sets
// bit 0 of *overflow, fewer than k_min candidates in all (a floor that too
// few rows cleared) bit 1.  One block per query: the radix select of topk_rows_kernel on
// the keys themselves, then a bitonic sort by key.
__global__ void __launch_bounds__(TOPK_THREADS)
    select_keys_kernel(const uint64_t* __restrict__ cand, const int32_t* __restrict__ count,
                       int32_t splits, int64_t nq_pad, int32_t cap, int64_t nq, int32_t k,
                       int32_t k_min, uint64_t* __restrict__ out,
                       int32_t* __restrict__ overflow) {
  constexpr int WARPS = TOPK_THREADS / 32;
  __shared__ uint32_t hist[WARPS][256];
  __shared__ uint32_t suffix[256];
  __shared__ uint32_t offs[129];
  __shared__ unsigned long long s_prefix;
  __shared__ uint32_t s_need, s_done;
  __shared__ uint32_t taken_above, taken_equal;
  __shared__ unsigned long long sel[TOPK_KMAX];
  const int lid = threadIdx.x;
  const int warp = lid >> 5;
  const int64_t q = blockIdx.x;
  if (q >= nq) return;
  // prefix offsets of the buffers' candidate runs (splits <= 128)
  if (lid == 0) {
    uint32_t acc = 0;
    bool over = false;
    for (int sp = 0; sp < splits; ++sp) {
      offs[sp] = acc;
      const int32_t c = count[(size_t)sp * nq_pad + q];
      over |= c > cap;
      acc += (uint32_t)(c < cap ? c : cap);
    }
    offs[splits] = acc;
    if (over) atomicOr(overflow, 1);
    if (acc < (uint32_t)k_min) atomicOr(overflow, 2);
  }
  __syncthreads();
  const uint32_t total = offs[splits];
  const uint32_t keff = (uint32_t)k < total ? (uint32_t)k : total;
  auto cand_at = [&](uint32_t i) -> uint64_t {
    // the last buffer whose run starts at or before i (runs may be empty)
    int lo = 0, hi = splits - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (offs[mid] <= i) lo = mid; else hi = mid - 1;
    }
    return cand[((size_t)lo * nq_pad + q) * cap + (i - offs[lo])];
  };
  uint64_t prefix = 0, mask = 0;
  uint32_t need = keff;
  if (keff > 0) {
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int i = lid; i < WARPS * 256; i += TOPK_THREADS) (&hist[0][0])[i] = 0u;
      __syncthreads();
      for (uint32_t i = lid; i < total; i += TOPK_THREADS) {
        const uint64_t key = cand_at(i);
        if ((key & mask) == prefix) atomicAdd(&hist[warp][(uint32_t)(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      uint32_t c = 0;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) c += hist[w][lid];
      suffix[lid] = c;
      __syncthreads();
      for (int off = 1; off < 256; off <<= 1) {
        const uint32_t add = lid + off < 256 ? suffix[lid + off] : 0u;
        __syncthreads();
        suffix[lid] += add;
        __syncthreads();
      }
      const uint32_t at_or_above = suffix[lid];
      const uint32_t above = at_or_above - c;
      if (at_or_above >= need && above < need) {
        s_prefix = prefix | ((uint64_t)lid << shift);
        s_need = need - above;
        s_done = (c == need - above) ? 1u : 0u;
      }
      __syncthreads();
      prefix = s_prefix;
      need = s_need;
      mask |= 255ull << shift;
      const bool done = s_done != 0;
      __syncthreads();
      if (done) break;
    }
  }
  if (lid == 0) {
    taken_above = 0;
    taken_equal = 0;
  }
  for (int i = lid; i < TOPK_KMAX; i += TOPK_THREADS) sel[i] = 0ull;
  __syncthreads();
  const uint32_t n_above = keff - need;
  if (keff > 0) {
    for (uint32_t i = lid; i < total; i += TOPK_THREADS) {
      const uint64_t key = cand_at(i);
      const uint64_t mk = key & mask;
      if (mk > prefix) {
        sel[atomicAdd(&taken_above, 1u)] = key;
      } else if (mk == prefix) {
        const uint32_t at = atomicAdd(&taken_equal, 1u);
        if (at < need) sel[n_above + at] = key;
      }
    }
  }
  __syncthreads();
  uint32_t size_pow2 = 1;
  while (size_pow2 < keff) size_pow2 <<= 1;
  for (uint32_t size = 2; size <= size_pow2; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t i = lid; i < size_pow2; i += TOPK_THREADS) {
        const uint32_t j = i ^ stride;
        if (j > i) {
          const bool forward = (i & size) == 0;
          const uint64_t a = sel[i], b = sel[j];
          if (forward != (a > b)) {
            sel[i] = b;
            sel[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = lid; i < k; i += TOPK_THREADS) out[(size_t)q * k + i] = (uint32_t)i < keff ? sel[i] : 0ull;
}

struct RefineParams {
  const float* dataset;       // [n][d]
  int64_t n;
  int32_t d;
  const float* queries;       // [nq][d]
  int64_t nq;
  const int32_t* candidates;  // [nq][c]
  int32_t c;
  int32_t metric;             // 0 inner product, 1 L2, 2 cosine
  float* scores;              // [nq][c]: larger is closer, -inf where invalid
};

// One warp per REFINE_ROWS (query, candidate) pairs: the exact score of each
// candidate row as the reference computes it (src/ivf.cpp:1677-1690): L2
// -sum((r - q)^2), inner product sum(r q), cosine on rows and query divided
// by max(norm, 1e-30).  Ids outside [0, n) score -inf.  The rows' loads are
// issued together (a gather is latency-bound: one 512-byte row per warp
// leaves most of the memory system idle); each pair's sum runs in the same
// order as with one pair per warp.
constexpr int REFINE_ROWS = 4;

__global__ void refine_scores_kernel(RefineParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t total = p.nq * (int64_t)p.c;
  const int64_t first =
      ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * REFINE_ROWS;
  if (first >= total) return;
  const float* r[REFINE_ROWS];
  const float* x[REFINE_ROWS];
  bool on[REFINE_ROWS], valid[REFINE_ROWS];
#pragma unroll
  for (int t = 0; t < REFINE_ROWS; ++t) {
    const int64_t pair = first + t;
    on[t] = pair < total;
    const int32_t id = on[t] ? p.candidates[pair] : -1;
    valid[t] = on[t] && id >= 0 && (int64_t)id < p.n;
    r[t] = p.dataset + (valid[t] ? (int64_t)id * p.d : 0);
    x[t] = p.queries + (on[t] ? pair / p.c : 0) * p.d;
  }
  float acc[REFINE_ROWS], rr[REFINE_ROWS], xx[REFINE_ROWS];
#pragma unroll
  for (int t = 0; t < REFINE_ROWS; ++t) acc[t] = rr[t] = xx[t] = 0.0f;
  for (int j = lane; j < p.d; j += 32) {
    float a[REFINE_ROWS], bq[REFINE_ROWS];
#pragma unroll
    for (int t = 0; t < REFINE_ROWS; ++t) {
      a[t] = valid[t] ? __ldg(r[t] + j) : 0.0f;
      bq[t] = valid[t] ? __ldg(x[t] + j) : 0.0f;
    }
#pragma unroll
    for (int t = 0; t < REFINE_ROWS; ++t) {
      if (p.metric == 1) {
        const float df = a[t] - bq[t];
        acc[t] = fmaf(df, df, acc[t]);
      } else {
        acc[t] = fmaf(a[t], bq[t], acc[t]);
        if (p.metric == 2) {
          rr[t] = fmaf(a[t], a[t], rr[t]);
          xx[t] = fmaf(bq[t], bq[t], xx[t]);
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < REFINE_ROWS; ++t) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], off);
      if (p.metric == 2) {
        rr[t] += __shfl_xor_sync(0xffffffffu, rr[t], off);
        xx[t] += __shfl_xor_sync(0xffffffffu, xx[t], off);
      }
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int t = 0; t < REFINE_ROWS; ++t) {
      if (!on[t]) continue;
      float sc;
      if (!valid[t]) {
        sc = -INFINITY;
      } else if (p.metric == 1) {
        sc = -acc[t];
      } else if (p.metric == 2) {
        sc = acc[t] / (fmaxf(sqrtf(rr[t]), 1e-30f) * fmaxf(sqrtf(xx[t]), 1e-30f));
      } else {
        sc = acc[t];
      }
      p.scores[first + t] = sc;
    }
  }
}

// Selected positions -> candidate ids and distances; infinite scores are
// missing (-1, +inf for L2, -inf otherwise), as src/ivf.cpp:1694-1699.
__global__ void refine_finish_kernel(const int32_t* __restrict__ candidates, int32_t c,
                                     int64_t count, int32_t k, int32_t l2,
                                     int32_t* __restrict__ ids, float* __restrict__ dist) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= count) return;
  const int64_t q = i / k;
  const int32_t pos = ids[i];
  const float s = dist[i];
  const bool missing = pos < 0 || isinf(s);
  ids[i] = missing ? -1 : candidates[q * c + pos];
  dist[i] = l2 ? (missing ? INFINITY : -s) : (missing ? -INFINITY : s);
}

}  // namespace mlxvs_b200
