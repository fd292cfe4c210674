// Fused distance GEMM + top-k selection for sm_100a (the B200 replacement of
// the reference's per-tile mx::matmul + L2 transform + mlxvs_topk_merge,
// src/knn.cpp:104-121 and src/kernels.h:37-229).
//
// One CTA (persistent, one per SM) works through "units": a block of QB
// queries against a contiguous range of base tiles of BN = 256 rows.
//   warp EW      TMA producer: query block (once per unit, or per K chunk when
//                the block does not fit in shared memory) and base chunks of
//                64 fp16 columns into a ring of shared-memory stages.
//   warp EW + 1  allocates 512 TMEM columns (two 128 x 256 fp32
//                accumulators) and issues tcgen05.mma (M=128, N=256, K=16).
//   warps 0..EW-1 epilogue, one thread per query (TMEM lane): loads its
//                256 scores per tile with tcgen05.ld, subtracts the per-row
//                term (|b|^2 for L2, +inf on padding rows), and keeps the
//                k best (score, id) keys in a min-heap in shared memory.
//                A tile is rejected with one compare when its best score is
//                below the query's floor: the heap's worst key or, better,
//                the floor shared by the other units of the same query
//                through a global atomicMax (any unit's k-th best is a lower
//                bound of the final k-th best).
// The full Q x N score matrix never reaches global memory: each unit writes
// only its k keys per query to the partial lists, merged by merge_keys.
//
// NPASS = 1: operands are the inputs themselves in fp16 (used only when
// every input value is exactly an fp16, e.g. the integer-valued benchmark
// data): products are exact and accumulate in fp32, as the reference's
// float32 matmul.  NPASS = 3: split fp16 (x = hi + lo, power-of-two scaled),
// D = Ahi*Bhi + Ahi*Blo + Alo*Bhi: about 22 significant bits per product.
#pragma once

#include "common.cuh"

namespace mlxvs_b200 {

constexpr int GT_BN = 256;       // base rows per tile (MMA N)
constexpr int GT_KCH = 64;       // fp16 columns per K chunk (one 128-byte swizzle row)
constexpr int GT_ACHUNK = 128 * 128;  // bytes of one A chunk (128 rows x 128 B)
constexpr int GT_BCHUNK = GT_BN * 128;  // bytes of one B chunk
constexpr int GT_SHARE_TILES = 4;  // tiles between exchanges of the shared floor

struct KnnGemmParams {
  int32_t qblocks;   // query blocks of QB rows
  int32_t tiles;     // base tiles of GT_BN rows
  int32_t splits;    // base tile ranges per query block
  int32_t units;     // qblocks * splits
  int32_t kchunks;   // padded dimension / 64
  int32_t k;         // neighbors kept, <= heap capacity
  int32_t stages;    // depth of the base-chunk ring
  int32_t a_stream;  // 1: query chunks travel with the base chunks
  int64_t n_valid;   // base rows
  int64_t nq;        // queries
  int64_t nq_pad;    // query rows of the partial lists (multiple of QB)
  int64_t id_offset;
  const float* nb;                 // [tiles * GT_BN]: subtracted from each dot
  uint64_t* partial;               // [splits][nq_pad][k] keys
  unsigned long long* gfloor;      // [nq_pad] shared floor keys (0 = none)
  float out_scale;                 // partial scores are written as score * out_scale
  uint32_t* err;                   // error word (bounded waits that gave up)
  uint64_t wait_ns;                // limit of every wait
};

template <int QB, int NPASS>
struct GemmLayout {
  static constexpr int EW = QB >= 32 ? QB / 32 : 1;  // epilogue warps
  static constexpr int THREADS = (EW + 2) * 32;
  static constexpr int NPA = NPASS == 1 ? 1 : 2;  // operand planes: hi (, lo)
};

// Shared-memory offsets, computed identically on host and device.
struct GemmSmem {
  uint32_t a_off, a_bytes;      // resident query block (0 bytes when streamed)
  uint32_t stage_off, stage_bytes;
  uint32_t heap_off, heap_bytes;
  uint32_t bar_off;
  uint32_t total;
};

__host__ __device__ inline GemmSmem gemm_smem(int QB, int npa, int kchunks, int stages,
                                              int a_stream, int k) {
  GemmSmem s;
  s.a_off = 0;
  s.a_bytes = a_stream ? 0u : (uint32_t)(npa * kchunks * GT_ACHUNK);
  s.stage_off = s.a_off + s.a_bytes;
  s.stage_bytes = (uint32_t)(npa * (GT_BCHUNK + (a_stream ? GT_ACHUNK : 0)));
  s.heap_off = s.stage_off + (uint32_t)stages * s.stage_bytes;
  s.heap_bytes = (uint32_t)(QB * k * 8);
  s.bar_off = (s.heap_off + s.heap_bytes + 15u) & ~15u;
  // full[stages], empty[stages], a_full, a_empty, acc_full[2], acc_empty[2], aux
  s.total = s.bar_off + (uint32_t)(2 * stages + 7) * 8u + 16u;
  return s;
}

#ifdef __CUDACC__

// Replaces the root of a min-heap of k keys (slot s of this thread's heap at
// heap[s * QB]) by key, which is larger than the root.
template <int QB>
__device__ __forceinline__ void heap_replace_root(uint64_t* heap, int k, uint64_t key) {
  int i = 0;
  for (;;) {
    int l = 2 * i + 1;
    if (l >= k) break;
    uint64_t mv = heap[l * QB];
    int m = l;
    if (l + 1 < k) {
      uint64_t rv = heap[(l + 1) * QB];
      if (rv < mv) {
        mv = rv;
        m = l + 1;
      }
    }
    if (mv >= key) break;
    heap[i * QB] = mv;
    i = m;
  }
  heap[i * QB] = key;
}

struct EpiState {
  uint64_t floor;  // no candidate at or below this key can be in the result
  uint64_t gfl;    // last shared floor seen
  float thr;       // score of floor (-inf when none): the fast rejection test
};

// The slow path of a chunk whose best score reached the floor: every score of
// the chunk is tried against the heap.  Out of line (it is rare), the state
// passed and returned by value so that it stays in registers.
template <int QB>
__device__ __noinline__ EpiState epi_insert_chunk(const float (&v)[32], int64_t col0,
                                                  int64_t n_valid, int64_t id_offset,
                                                  uint64_t* heap, int k, EpiState st) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (v[j] >= st.thr && col0 + j < n_valid) {
      uint64_t key = make_key(v[j], (uint32_t)(id_offset + col0 + j));
      if (key > st.floor) {
        heap_replace_root<QB>(heap, k, key);
        uint64_t root = heap[0];
        st.floor = root > st.gfl ? root : st.gfl;
        st.thr = key_score(st.floor);
      }
    }
  }
  return st;
}

// Waits on the register outputs of the preceding tcgen05.ld so the compiler
// cannot read them before the load has completed.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

template <int QB>
__device__ __forceinline__ void epi_chunk(const uint32_t (&r)[32], const float* nbp, int64_t col0,
                                          const KnnGemmParams& p, uint64_t* heap,
                                          EpiState& st) {
  float v[32];
  const float4* nb4 = reinterpret_cast<const float4*>(nbp);
#pragma unroll
  for (int j4 = 0; j4 < 8; ++j4) {
    float4 t = __ldg(nb4 + j4);
    v[4 * j4 + 0] = __uint_as_float(r[4 * j4 + 0]) - t.x;
    v[4 * j4 + 1] = __uint_as_float(r[4 * j4 + 1]) - t.y;
    v[4 * j4 + 2] = __uint_as_float(r[4 * j4 + 2]) - t.z;
    v[4 * j4 + 3] = __uint_as_float(r[4 * j4 + 3]) - t.w;
  }
  float m[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) m[j] = fmaxf(v[j], v[j + 16]);
#pragma unroll
  for (int j = 0; j < 8; ++j) m[j] = fmaxf(m[j], m[j + 8]);
#pragma unroll
  for (int j = 0; j < 4; ++j) m[j] = fmaxf(m[j], m[j + 4]);
  float mx = fmaxf(fmaxf(m[0], m[2]), fmaxf(m[1], m[3]));
  if (mx >= st.thr && (QB >= 32 || (threadIdx.x & 31) < QB))
    st = epi_insert_chunk<QB>(v, col0, p.n_valid, p.id_offset, heap, p.k, st);
}

template <int QB, int NPASS>
__global__ void __launch_bounds__(GemmLayout<QB, NPASS>::THREADS, 1)
    knn_gemm_topk_kernel(const __grid_constant__ CUtensorMap tm_a_hi,
                         const __grid_constant__ CUtensorMap tm_a_lo,
                         const __grid_constant__ CUtensorMap tm_b_hi,
                         const __grid_constant__ CUtensorMap tm_b_lo, const KnnGemmParams p) {
  using L = GemmLayout<QB, NPASS>;
  constexpr int EW = L::EW;
  constexpr int NPA = L::NPA;
  constexpr uint32_t IDESC = idesc_f16_f32(128, GT_BN);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const GemmSmem lay = gemm_smem(QB, NPA, p.kchunks, p.stages, p.a_stream, p.k);
  uint8_t* a_res = smem + lay.a_off;
  uint8_t* stage_base = smem + lay.stage_off;
  uint64_t* heap_all = reinterpret_cast<uint64_t*>(smem + lay.heap_off);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + lay.bar_off);
  uint64_t* full = bars;
  uint64_t* empty = bars + p.stages;
  uint64_t* a_full = bars + 2 * p.stages;
  uint64_t* a_empty = a_full + 1;
  uint64_t* acc_full = a_full + 2;
  uint64_t* acc_empty = a_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(a_full + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EW);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == EW + 1) {
    tmem_alloc(tmem_slot, 2 * GT_BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == EW) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      tma_prefetch_desc(&tm_a_hi);
      tma_prefetch_desc(&tm_b_hi);
      if (NPASS == 3) {
        tma_prefetch_desc(&tm_a_lo);
        tma_prefetch_desc(&tm_b_lo);
      }
      const uint32_t a_bytes = (uint32_t)(NPA * QB * 128);  // per K chunk
      uint32_t stage = 0, phase = 0, uidx = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uidx) {
        const int qb = u % p.qblocks;
        const int split = u / p.qblocks;
        const int t0 = (int)((int64_t)split * p.tiles / p.splits);
        const int t1 = (int)((int64_t)(split + 1) * p.tiles / p.splits);
        if (!p.a_stream) {
          if (uidx > 0 && !mbar_wait(a_empty, (uidx - 1) & 1, abort_flag, p.wait_ns)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(a_full, a_bytes * p.kchunks);
          for (int kc = 0; kc < p.kchunks; ++kc) {
            tma_load_2d(a_res + (size_t)kc * GT_ACHUNK, &tm_a_hi, a_full, kc * GT_KCH, qb * QB);
            if (NPASS == 3)
              tma_load_2d(a_res + (size_t)(p.kchunks + kc) * GT_ACHUNK, &tm_a_lo, a_full,
                          kc * GT_KCH, qb * QB);
          }
        }
        for (int t = t0; t < t1 && ok; ++t) {
          for (int kc = 0; kc < p.kchunks; ++kc) {
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.wait_ns)) {
              ok = false;
              break;
            }
            uint8_t* st = stage_base + (size_t)stage * lay.stage_bytes;
            mbar_arrive_expect_tx(&full[stage],
                                  (uint32_t)(NPA * GT_BCHUNK) + (p.a_stream ? a_bytes : 0u));
            tma_load_2d(st, &tm_b_hi, &full[stage], kc * GT_KCH, t * GT_BN);
            if (NPASS == 3) tma_load_2d(st + GT_BCHUNK, &tm_b_lo, &full[stage], kc * GT_KCH, t * GT_BN);
            if (p.a_stream) {
              uint8_t* sa = st + NPA * GT_BCHUNK;
              tma_load_2d(sa, &tm_a_hi, &full[stage], kc * GT_KCH, qb * QB);
              if (NPASS == 3) tma_load_2d(sa + GT_ACHUNK, &tm_a_lo, &full[stage], kc * GT_KCH, qb * QB);
            }
            if (++stage == (uint32_t)p.stages) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(p.err, ERR_WAIT_PRODUCER);
      }
      // Every load issued lands before the CTA may exit: the last arm of each
      // stage completes by itself (bounded wait all the same).
      for (int s = 0; s < p.stages; ++s) {
        // the stage's most recent arm had parity (phase of that arm)
        uint32_t par = ((uint32_t)s < stage) ? phase : (phase ^ 1);
        mbar_wait(&full[s], par, abort_flag, p.wait_ns);
      }
    }
  } else if (warp == EW + 1) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, acc = 0, acc_ph = 0, uidx = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uidx) {
        const int split = u / p.qblocks;
        const int t0 = (int)((int64_t)split * p.tiles / p.splits);
        const int t1 = (int)((int64_t)(split + 1) * p.tiles / p.splits);
        if (!p.a_stream) {
          if (!mbar_wait(a_full, uidx & 1, abort_flag, p.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        for (int t = t0; t < t1 && ok; ++t) {
          if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1, abort_flag, p.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * GT_BN;
          for (int kc = 0; kc < p.kchunks; ++kc) {
            if (!mbar_wait(&full[stage], phase, abort_flag, p.wait_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            uint8_t* st = stage_base + (size_t)stage * lay.stage_bytes;
            const uint32_t b_hi = smem_u32(st);
            const uint32_t b_lo = b_hi + GT_BCHUNK;
            uint32_t a_hi, a_lo;
            if (p.a_stream) {
              a_hi = b_hi + NPA * GT_BCHUNK;
              a_lo = a_hi + GT_ACHUNK;
            } else {
              a_hi = smem_u32(a_res) + (uint32_t)kc * GT_ACHUNK;
              a_lo = smem_u32(a_res) + (uint32_t)(p.kchunks + kc) * GT_ACHUNK;
            }
#pragma unroll
            for (int kk = 0; kk < GT_KCH / 16; ++kk) {
              const uint32_t acc_in = (kc | kk) != 0;
              umma_f16_ss(d_tmem, sdesc_k128(a_hi + kk * 32), sdesc_k128(b_hi + kk * 32), IDESC,
                          acc_in);
              if (NPASS == 3) {
                umma_f16_ss(d_tmem, sdesc_k128(a_hi + kk * 32), sdesc_k128(b_lo + kk * 32),
                            IDESC, 1u);
                umma_f16_ss(d_tmem, sdesc_k128(a_lo + kk * 32), sdesc_k128(b_hi + kk * 32),
                            IDESC, 1u);
              }
            }
            umma_commit(&empty[stage]);
            if (++stage == (uint32_t)p.stages) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          umma_commit(&acc_full[acc]);
          acc ^= 1;
          if (acc == 0) acc_ph ^= 1;
        }
        if (!p.a_stream) umma_commit(a_empty);
      }
      if (!ok) {
        *abort_flag = 1;
        atomicOr(p.err, ERR_WAIT_MMA);
      }
      // let every issued MMA finish before the columns are freed
      umma_commit(a_empty);
      mbar_wait(a_empty, (p.a_stream ? 0u : uidx) & 1, abort_flag, p.wait_ns);
    }
  } else {
    // ------------------------------------------------------------- epilogue
    const int row = warp * 32 + lane;  // TMEM lane = query within the block
    // with QB < 32 the lanes past QB only join the warp-collective loads
    const bool row_on = row < QB;
    uint64_t* heap = heap_all + (row_on ? row : 0);
    uint32_t acc = 0, acc_ph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
      const int qb = u % p.qblocks;
      const int split = u / p.qblocks;
      const int t0 = (int)((int64_t)split * p.tiles / p.splits);
      const int t1 = (int)((int64_t)(split + 1) * p.tiles / p.splits);
      const int64_t q = (int64_t)qb * QB + row;
      const bool q_ok = row_on && q < p.nq;
      if (row_on)
        for (int s = 0; s < p.k; ++s) heap[s * QB] = 0;
      EpiState st;
      st.gfl = q_ok ? *reinterpret_cast<volatile unsigned long long*>(p.gfloor + q) : 0ull;
      st.floor = st.gfl;
      st.thr = key_score(st.floor);
      for (int t = t0; t < t1; ++t) {
        if (!mbar_wait(&acc_full[acc], acc_ph, abort_flag, p.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(warp * 32) << 16) + acc * GT_BN;
        const int64_t col_base = (int64_t)t * GT_BN;
        const float* nbp = p.nb + col_base;
        uint32_t ra[32], rb[32];
        tmem_ld32(taddr, ra);
        tmem_wait_ld_regs(ra);
#pragma unroll 1
        for (int c = 0; c < GT_BN / 32; c += 2) {
          // tcgen05.ld is warp-collective: reconverge after a divergent slow path
          __syncwarp();
          tmem_ld32(taddr + (c + 1) * 32, rb);
          epi_chunk<QB>(ra, nbp + c * 32, col_base + c * 32, p, heap, st);
          __syncwarp();
          tmem_wait_ld_regs(rb);
          if (c + 2 < GT_BN / 32) tmem_ld32(taddr + (c + 2) * 32, ra);
          epi_chunk<QB>(rb, nbp + (c + 1) * 32, col_base + (c + 1) * 32, p, heap, st);
          __syncwarp();
          if (c + 2 < GT_BN / 32) tmem_wait_ld_regs(ra);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
        if (q_ok && ((t - t0) % GT_SHARE_TILES) == GT_SHARE_TILES - 1) {
          const uint64_t root = heap[0];
          uint64_t g;
          if (root != 0) {
            g = atomicMax(p.gfloor + q, (unsigned long long)root);
            if (root > g) g = root;
          } else {
            g = *reinterpret_cast<volatile unsigned long long*>(p.gfloor + q);
          }
          if (g > st.gfl) {
            st.gfl = g;
            if (g > st.floor) {
              st.floor = g;
              st.thr = key_score(g);
            }
          }
        }
      }
      if (!ok) break;
      if (row_on && q < p.nq_pad) {
        uint64_t* out = p.partial + ((size_t)split * p.nq_pad + q) * p.k;
        for (int s = 0; s < p.k; ++s) {
          uint64_t key = heap[s * QB];
          if (key != 0 && p.out_scale != 1.0f)
            key = make_key(key_score(key) * p.out_scale, ~(uint32_t)key);
          out[s] = key;
        }
      }
    }
    if (!ok) {
      *abort_flag = 1;
      atomicOr(p.err, ERR_WAIT_EPILOGUE);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == EW + 1) tmem_dealloc(tmem_base, 2 * GT_BN);
}

#endif  // __CUDACC__

}  // namespace mlxvs_b200
