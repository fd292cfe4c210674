// Exact Hamming k-NN scan for sm_100a: XOR + popcount of packed codes with
// the top-k selection fused in (replaces the reference's
// IVF_BINARY_SCAN_SOURCE, src/ivf_kernels.h:549-595, driven as an
// all-lists scan by src/ivf.cpp:1343-1403, plus its finish / argsort merges).
//
// One CTA works through units (a block of QH queries x a range of base tiles
// of HT rows), like the distance GEMM:
//   warp QH/32     producer: copies each tile of HT contiguous codes
//                  (HT * 16V bytes) into a shared-memory ring with one
//                  cp.async.bulk (the TMA engine), completion on an mbarrier.
//   warps 0..      one thread per query, its code in 4V registers; every
//                  thread reads each row of the tile as V 128-bit shared
//                  loads (a broadcast) and adds popc(q ^ row) over 4V words.
// Selection is the GEMM epilogue's: a min-heap of (score = -distance, id)
// keys per query in shared memory, a one-compare rejection against the
// query's floor, floors shared across units by atomicMax.
#pragma once

#include "common.cuh"

namespace mlxvs_b200 {

constexpr int HM_HT = 128;  // base codes per tile
constexpr int HM_SHARE_TILES = 8;

struct HammingParams {
  const uint8_t* rows;      // [n][16 V] codes, 16-byte aligned
  const uint8_t* queries;   // [nq][16 V]
  int64_t n;
  int64_t nq;
  int64_t nq_pad;
  int32_t qblocks;
  int32_t tiles;
  int32_t splits;
  int32_t units;
  int32_t k;
  int32_t stages;
  int64_t id_offset;
  uint64_t* partial;             // [splits][nq_pad][k]
  unsigned long long* gfloor;    // [nq_pad]
  uint32_t* err;
  uint64_t wait_ns;
};

__host__ __device__ inline uint32_t hamming_smem_bytes(int V, int QH, int k, int stages) {
  uint32_t ring = (uint32_t)stages * HM_HT * 16u * (uint32_t)V;
  uint32_t heap = (uint32_t)QH * (uint32_t)k * 8u;
  return ring + heap + (uint32_t)(2 * stages + 2) * 8u + 16u;
}

#ifdef __CUDACC__

template <int QH>
__device__ __forceinline__ void hm_heap_replace_root(uint64_t* heap, int k, uint64_t key) {
  int i = 0;
  for (;;) {
    int l = 2 * i + 1;
    if (l >= k) break;
    uint64_t mv = heap[l * QH];
    int m = l;
    if (l + 1 < k) {
      uint64_t rv = heap[(l + 1) * QH];
      if (rv < mv) {
        mv = rv;
        m = l + 1;
      }
    }
    if (mv >= key) break;
    heap[i * QH] = mv;
    i = m;
  }
  heap[i * QH] = key;
}

template <int QH>
__device__ __forceinline__ void hm_insert(uint32_t dist, uint32_t id, uint64_t* heap, int k,
                                       uint64_t& floor, uint64_t gfl, uint32_t& thr) {
  uint64_t key = make_key(-(float)dist, id);
  if (key > floor) {
    hm_heap_replace_root<QH>(heap, k, key);
    uint64_t root = heap[0];
    floor = root > gfl ? root : gfl;
    thr = (uint32_t)(-key_score(floor));
  }
}

template <int V, int QH>
__global__ void __launch_bounds__(QH + 32)
    hamming_topk_kernel(const HammingParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t tile_bytes = HM_HT * 16u * V;
  uint8_t* ring = smem;
  uint64_t* heap_all = reinterpret_cast<uint64_t*>(smem + (size_t)p.stages * tile_bytes);
  uint64_t* bars = heap_all + (size_t)QH * p.k;
  uint64_t* full = bars;
  uint64_t* empty = bars + p.stages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * p.stages + 2);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr int CW = QH / 32;  // consumer warps

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CW);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == CW) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
        const int split = u / p.qblocks;
        const int t0 = (int)((int64_t)split * p.tiles / p.splits);
        const int t1 = (int)((int64_t)(split + 1) * p.tiles / p.splits);
        for (int t = t0; t < t1; ++t) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.wait_ns)) {
            ok = false;
            break;
          }
          int64_t r0 = (int64_t)t * HM_HT;
          int64_t rows_t = p.n - r0 < HM_HT ? p.n - r0 : HM_HT;
          uint32_t bytes = (uint32_t)rows_t * 16u * V;
          mbar_arrive_expect_tx(&full[stage], bytes);
          bulk_load(ring + (size_t)stage * tile_bytes, p.rows + (size_t)r0 * 16 * V, bytes,
                    &full[stage]);
          if (++stage == (uint32_t)p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(p.err, ERR_WAIT_PRODUCER);
      }
      for (int s = 0; s < p.stages; ++s) {
        uint32_t par = ((uint32_t)s < stage) ? phase : (phase ^ 1);
        mbar_wait(&full[s], par, abort_flag, p.wait_ns);
      }
    }
  } else {
    const int row = threadIdx.x;
    uint64_t* heap = heap_all + row;
    uint32_t stage = 0, phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
      const int qb = u % p.qblocks;
      const int split = u / p.qblocks;
      const int t0 = (int)((int64_t)split * p.tiles / p.splits);
      const int t1 = (int)((int64_t)(split + 1) * p.tiles / p.splits);
      const int64_t q = (int64_t)qb * QH + row;
      const bool q_ok = q < p.nq;
      uint4 qv[V];
      const uint4* qsrc = reinterpret_cast<const uint4*>(p.queries + (size_t)(q_ok ? q : 0) * 16 * V);
#pragma unroll
      for (int w = 0; w < V; ++w) qv[w] = q_ok ? __ldg(qsrc + w) : make_uint4(0u, 0u, 0u, 0u);
      for (int s = 0; s < p.k; ++s) heap[s * QH] = 0;
      uint64_t gfl = q_ok ? *reinterpret_cast<volatile unsigned long long*>(p.gfloor + q) : 0ull;
      uint64_t floor = gfl;
      uint32_t thr = floor ? (uint32_t)(-key_score(floor)) : 0xFFFFFFFFu;
      for (int t = t0; t < t1; ++t) {
        if (!mbar_wait(&full[stage], phase, abort_flag, p.wait_ns)) {
          ok = false;
          break;
        }
        const int64_t r0 = (int64_t)t * HM_HT;
        const int rows_t = (int)(p.n - r0 < HM_HT ? p.n - r0 : HM_HT);
        const uint4* tile = reinterpret_cast<const uint4*>(ring + (size_t)stage * tile_bytes);
        int r = 0;
        for (; r + 2 <= rows_t; r += 2) {
          uint32_t a0 = 0, a1 = 0;
#pragma unroll
          for (int w = 0; w < V; ++w) {
            uint4 b0 = tile[r * V + w];
            uint4 b1 = tile[(r + 1) * V + w];
            a0 += __popc(b0.x ^ qv[w].x) + __popc(b0.y ^ qv[w].y) + __popc(b0.z ^ qv[w].z) +
                  __popc(b0.w ^ qv[w].w);
            a1 += __popc(b1.x ^ qv[w].x) + __popc(b1.y ^ qv[w].y) + __popc(b1.z ^ qv[w].z) +
                  __popc(b1.w ^ qv[w].w);
          }
          if (a0 <= thr) hm_insert<QH>(a0, (uint32_t)(p.id_offset + r0 + r), heap, p.k, floor, gfl, thr);
          if (a1 <= thr) hm_insert<QH>(a1, (uint32_t)(p.id_offset + r0 + r + 1), heap, p.k, floor, gfl, thr);
        }
        for (; r < rows_t; ++r) {
          uint32_t a0 = 0;
#pragma unroll
          for (int w = 0; w < V; ++w) {
            uint4 b0 = tile[r * V + w];
            a0 += __popc(b0.x ^ qv[w].x) + __popc(b0.y ^ qv[w].y) + __popc(b0.z ^ qv[w].z) +
                  __popc(b0.w ^ qv[w].w);
          }
          if (a0 <= thr) hm_insert<QH>(a0, (uint32_t)(p.id_offset + r0 + r), heap, p.k, floor, gfl, thr);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == (uint32_t)p.stages) {
          stage = 0;
          phase ^= 1;
        }
        if (q_ok && ((t - t0) % HM_SHARE_TILES) == HM_SHARE_TILES - 1) {
          const uint64_t root = heap[0];
          uint64_t g;
          if (root != 0) {
            g = atomicMax(p.gfloor + q, (unsigned long long)root);
            if (root > g) g = root;
          } else {
            g = *reinterpret_cast<volatile unsigned long long*>(p.gfloor + q);
          }
          if (g > gfl) {
            gfl = g;
            if (g > floor) {
              floor = g;
              thr = (uint32_t)(-key_score(floor));
            }
          }
        }
      }
      if (!ok) break;
      uint64_t* out = p.partial + ((size_t)split * p.nq_pad + q) * p.k;
      for (int s = 0; s < p.k; ++s) out[s] = heap[s * QH];
    }
    if (!ok) {
      *abort_flag = 1;
      atomicOr(p.err, ERR_WAIT_EPILOGUE);
    }
  }
  __syncthreads();
}

// Bit-packed codes [rows][bytes] -> +-1 int8 rows [rows_pad][d_pad] for the
// tensor-core path: bit j of byte b is dimension 8 b + j, a 1 bit is +1 and
// a 0 bit -1, and dimensions past the code and padding rows are 0.  The dot
// of two such rows is then bits - 2 * (their Hamming distance), exactly.
// One thread per two source bytes (16 output bytes).
__global__ void hamming_unpack_kernel(const uint8_t* __restrict__ src, int64_t rows,
                                      int64_t rows_pad, int32_t bytes, int32_t d_pad,
                                      int8_t* __restrict__ dst) {
  const int32_t pairs = d_pad / 16;
  const int64_t total = rows_pad * pairs;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / pairs;
    const int32_t b0 = (int32_t)(i - r * pairs) * 2;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (r < rows) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (b0 + h < bytes) {
          const uint32_t byte = src[r * bytes + b0 + h];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t v = ((byte >> j) & 1u) ? 0x01u : 0xFFu;
            w[h * 2 + (j >> 2)] |= v << (8 * (j & 3));
          }
        }
      }
    }
    *reinterpret_cast<uint4*>(dst + r * d_pad + (int64_t)b0 * 8) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

#endif  // __CUDACC__

}  // namespace mlxvs_b200
