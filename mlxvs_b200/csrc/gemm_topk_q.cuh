// Fused distance GEMM + top-k with a queued epilogue (sm_100a).
//
// The same units, TMA ring and tcgen05 MMA as knn_gemm_topk_kernel
// (gemm_topk.cuh), but the epilogue is split in two warp roles that meet in
// shared-memory queues, so the slow part of top-k selection never holds a
// TMEM accumulator:
//
//   filter warps 0..7   warp w reads TMEM lane quarter w % 4 and column half
//                       w / 4 of each 128 x 256 accumulator (tcgen05.ld), one
//                       query per lane.  Per 16 scores it takes the max and
//                       compares it with the query's threshold; a 16-score
//                       chunk that reaches it is copied into the query's
//                       queue for that column half (about 12 instructions),
//                       and the accumulator is released as soon as its last
//                       columns are in registers.
//   select warps 8..11  warp 8 + r owns queries 32 r .. 32 r + 31, one per
//                       lane, and holds each query's k best keys as one
//                       sorted register list covering both column halves.
//                       Every lane takes the next chunk of each of its
//                       query's two queues, and the warp inserts the chunks'
//                       candidates (two per lane per round, all lanes at
//                       once, one merge network for the pair); the
//                       list's worst key is the query's floor, published to
//                       the filter warps and the relay warp through shared
//                       memory.
//   warp 12             TMA producer (as in the inline kernel).
//   warp 13             TMEM allocation and MMA issue (as in the inline kernel).
//   warp 14             floor relay: publishes each query's list floor to the
//                       global shared floor (atomicMax) and brings the other
//                       units' floors back into shared memory, so that the
//                       filter and select loops never touch global memory
//                       between a unit's start and its end (a CTA-scope fence
//                       there would wait for the outstanding global access).
//
// Why: with one query per lane a 32-lane warp takes a slow path whenever any
// of its 32 queries has a candidate, and at k = 10 on 10^5-10^6 rows that is
// a few percent of all chunks however good the floors are; handled inline,
// each costs the filter a few hundred instructions on the path that frees
// the accumulator.  Queued, it costs the filter a copy, and the select warps
// batch the insertions of up to 32 queries per step on issue slots the
// filter leaves idle.
//
// MODE 1 (collect): the threshold is the fixed floor given in gfloor; the
// select warps append every candidate above it to the (split, column half,
// query) buffer instead of keeping a list.
//
// Queue protocol (single producer, single consumer per (column half, query)):
// the filter lane writes the chunk's 16 scores and first column into slot
// tail % QD, then advances tail with a release store; the select lane reads
// tail with an acquire load, reads the slot, and advances head with a
// release store once done with it.  A chunk with column -1 marks the end of
// the filter lane's unit.  Every wait is bounded.
#pragma once

#include "gemm_topk.cuh"

namespace mlxvs_b200 {

constexpr int QK_FILTER_WARPS = 8;
constexpr int QK_SELECT_WARPS = 4;
constexpr int QK_PRODUCER = QK_FILTER_WARPS + QK_SELECT_WARPS;  // warp 12
constexpr int QK_MMA = QK_PRODUCER + 1;                          // warp 13
constexpr int QK_FLOORS = QK_MMA + 1;                            // warp 14
constexpr int QK_THREADS = (QK_FLOORS + 1) * 32;                 // 480
constexpr int QK_QB = 128;                                       // queries per unit
// Select warps finish a unit at most 1 + QD units apart (a filter warp is
// at most QD end markers ahead of its select warp, and the filter warps are
// within two tiles of each other through the MMA's accumulators), so a ring
// of 8 per-unit counters (QD <= 4) tells the last of them apart.
constexpr int QK_END_RING = 8;
// A select warp with nothing queued sleeps between polls, from QK_NAP_MIN_NS
// doubling up to QK_NAP_MAX_NS: each poll is a few dozen instructions issued
// on an SM sub-partition that it shares with two filter warps and, on two of
// the four, with the TMA or the MMA warp, whose issue latency the tensor
// core feels directly.
#ifndef MLXVS_QK_NAP_MAX_NS
#define MLXVS_QK_NAP_MAX_NS 1024
#endif
constexpr uint32_t QK_NAP_MIN_NS = 32;
constexpr uint32_t QK_NAP_MAX_NS = MLXVS_QK_NAP_MAX_NS;
// The floor relay warp's interval between rounds.
#ifndef MLXVS_QK_RELAY_NAP_NS
#define MLXVS_QK_RELAY_NAP_NS 200
#endif
constexpr uint32_t QK_RELAY_NAP_NS = MLXVS_QK_RELAY_NAP_NS;

// Shared-memory layout of the queued kernel, computed identically on host
// and device.  The |b|^2 pieces of a tile travel with its first K chunk into
// a ring of their own, ceil(stages / kchunks) slots deep (a slot is free
// again once the stage that its tile's first chunk used has been released,
// by which time every MMA of that tile has completed).
struct QueuedSmem {
  uint32_t a_off, a_bytes;  // resident query block (0 when streamed)
  uint32_t ax_off;          // constant query-side block of the |b|^2 step
  uint32_t stage_off, stage_bytes;
  uint32_t x_off, x_slots;  // |b|^2 pieces ring
  uint32_t q_off;           // queues: scores [2][QD][4][128] float4, cols [2][QD][128]
  uint32_t qcol_off;
  uint32_t qtail_off, qhead_off;  // [2][128] u32 each
  uint32_t thr_off;               // [128] u64: (unit tag << 32) | threshold bits, the list's
  uint32_t gthr_off;              // [128] u64: the same for the other units' floors
  uint32_t misc_off;              // unit-end counters (a ring of QK_END_RING), units finished
  uint32_t bar_off;
  uint32_t total;
};

__host__ __device__ inline QueuedSmem queued_smem(int npa, int kchunks, int stages, int a_stream,
                                                  int extra, int qd) {
  QueuedSmem s;
  s.a_off = 0;
  s.a_bytes = a_stream ? 0u : (uint32_t)(npa * kchunks * GT_ACHUNK);
  s.ax_off = s.a_off + s.a_bytes;
  s.stage_off = s.ax_off + (extra ? (uint32_t)GT_AX : 0u);
  s.stage_bytes = (uint32_t)(npa * (GT_BCHUNK + (a_stream ? GT_ACHUNK : 0)));
  s.x_off = s.stage_off + (uint32_t)stages * s.stage_bytes;
  s.x_slots = extra ? (uint32_t)((stages + kchunks - 1) / kchunks) : 0u;
  s.q_off = s.x_off + s.x_slots * (uint32_t)GT_XCHUNK;
  s.qcol_off = s.q_off + (uint32_t)(2 * qd * 4 * QK_QB * 16);
  s.qtail_off = s.qcol_off + (uint32_t)(2 * qd * QK_QB * 4);
  s.qhead_off = s.qtail_off + 2u * QK_QB * 4u;
  s.thr_off = s.qhead_off + 2u * QK_QB * 4u;
  s.gthr_off = s.thr_off + (uint32_t)QK_QB * 8u;
  s.misc_off = s.gthr_off + (uint32_t)QK_QB * 8u;
  s.bar_off = s.misc_off + 4u * QK_END_RING + 16u;
  // full[stages], empty[stages], a_full, a_empty, acc_full[2], acc_empty[2], aux
  s.total = s.bar_off + (uint32_t)(2 * stages + 7) * 8u + 16u;
  return s;
}

#ifdef __CUDACC__

// Time limits inside the hot loops count SM cycles (clock64, a register
// read) instead of reading %globaltimer, which takes about a microsecond and
// would stall a select warp that polls its queues.  At most 2 GHz, a limit of
// 2 cycles per nanosecond lasts at least as long as the nanosecond limit.
__device__ __forceinline__ long long qk_cycle_limit(uint64_t limit_ns) {
  return (long long)(2 * limit_ns);
}

// Queue counters in shared memory with CTA-scope acquire / release order:
// the consumer's read of tail orders its reads of the slot after it, the
// producer's write of tail orders its writes of the slot before it, and the
// consumer's write of head orders its reads of the slot before it (cheaper
// than a full CTA fence around plain accesses).
__device__ __forceinline__ uint32_t qk_ld_acquire(const volatile uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];"
               : "=r"(v)
               : "r"((uint32_t)__cvta_generic_to_shared(const_cast<const uint32_t*>(p)))
               : "memory");
  return v;
}

__device__ __forceinline__ void qk_st_release(volatile uint32_t* p, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(const_cast<uint32_t*>(p))),
               "r"(v)
               : "memory");
}

// Copies one 16-score chunk into this lane's queue of its column half.
// Returns false when the wait for a free slot gave up (abort raised, or the
// time limit passed).
template <int QD>
__device__ __forceinline__ bool qk_push(const float* v, int32_t col, float4* qs, int32_t* qc,
                                        volatile uint32_t* tail_p, volatile uint32_t* head_p,
                                        uint32_t& tail, volatile int* abort, uint64_t limit_ns) {
  if (tail - *head_p >= (uint32_t)QD) {
    const long long start = clock64();
    for (uint32_t i = 1; tail - *head_p >= (uint32_t)QD; ++i) {
      if ((i & 63u) == 0) {
        if (*abort) return false;
        if (clock64() - start > qk_cycle_limit(limit_ns)) return false;
      }
    }
  }
  const uint32_t slot = tail % (uint32_t)QD;
  float4* dst = qs + (size_t)slot * 4 * QK_QB;
  if (v != nullptr) {
#pragma unroll
    for (int j4 = 0; j4 < 4; ++j4)
      dst[j4 * QK_QB] = make_float4(v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3]);
  }
  qc[slot * QK_QB] = col;
  qk_st_release(tail_p, ++tail);
  return true;
}

// The 16 scores r[o .. o + 15] as floats: raw fp32 dots, or s32 dots of
// +-1 codes turned into minus the Hamming distance (exact), minus the
// per-row terms nb[0 .. 15] when the accumulator is not the score (NBM 0).
template <int NBM, int OP>
__device__ __forceinline__ void qk_scores16(const uint32_t (&r)[32], int o, const float* nb,
                                            float dot_offset, float (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if constexpr (OP == 1)
      v[j] = fmaf(__int2float_rn((int32_t)r[o + j]), 0.5f, dot_offset);
    else
      v[j] = __uint_as_float(r[o + j]);
  }
  if constexpr (NBM == 0) {
    const float4* nb4 = reinterpret_cast<const float4*>(nb);
#pragma unroll
    for (int j4 = 0; j4 < 4; ++j4) {
      const float4 tt = __ldg(nb4 + j4);
      sub2(v[4 * j4 + 0], v[4 * j4 + 1], tt.x, tt.y);
      sub2(v[4 * j4 + 2], v[4 * j4 + 3], tt.z, tt.w);
    }
  }
}

__device__ __forceinline__ float qk_max16(const float (&v)[16]) {
  return max3(max3(max3(v[0], v[1], v[2]), max3(v[3], v[4], v[5]), max3(v[6], v[7], v[8])),
              max3(max3(v[9], v[10], v[11]), max3(v[12], v[13], v[14]), v[15]), -INFINITY);
}

// One filter step over 32 scores of this lane's query (raw accumulators r,
// columns col0 .. col0 + 31): the two 16-score maxima, one warp vote, and a
// copy into the queue of each 16-score half that reaches thr (its scores
// computed again there, so that only the maxima stay live).
template <int NBM, int OP, int QD>
__device__ __forceinline__ void qk_filter32(const uint32_t (&r)[32], const float* nb,
                                            int32_t col0, float thr, float dot_offset, float4* qs,
                                            int32_t* qc, volatile uint32_t* tail_p,
                                            volatile uint32_t* head_p, uint32_t& tail, bool& ok,
                                            volatile int* abort, uint64_t limit_ns) {
  float lo, hi;
  if constexpr (OP == 1 && NBM == 1) {
    // the score is increasing in the s32 dot: the max of the dots, converted
    int32_t m[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int32_t* x = reinterpret_cast<const int32_t*>(r) + 16 * h;
      const int32_t a0 = __vimax3_s32(x[0], x[1], x[2]), a1 = __vimax3_s32(x[3], x[4], x[5]);
      const int32_t a2 = __vimax3_s32(x[6], x[7], x[8]), a3 = __vimax3_s32(x[9], x[10], x[11]);
      const int32_t a4 = __vimax3_s32(x[12], x[13], x[14]);
      m[h] = __vimax3_s32(__vimax3_s32(a0, a1, a2), __vimax3_s32(a3, a4, x[15]), INT32_MIN);
    }
    lo = fmaf(__int2float_rn(m[0]), 0.5f, dot_offset);
    hi = fmaf(__int2float_rn(m[1]), 0.5f, dot_offset);
  } else {
    {
      float v[16];
      qk_scores16<NBM, OP>(r, 0, nb, dot_offset, v);
      lo = qk_max16(v);
    }
    {
      float v[16];
      qk_scores16<NBM, OP>(r, 16, nb + 16, dot_offset, v);
      hi = qk_max16(v);
    }
  }
  const bool a = lo >= thr, b = hi >= thr;
  if (__any_sync(0xffffffffu, a || b)) {
    if (a && ok) {
      float v[16];
      qk_scores16<NBM, OP>(r, 0, nb, dot_offset, v);
      ok = qk_push<QD>(v, col0, qs, qc, tail_p, head_p, tail, abort, limit_ns);
    }
    if (b && ok) {
      float v[16];
      qk_scores16<NBM, OP>(r, 16, nb + 16, dot_offset, v);
      ok = qk_push<QD>(v, col0 + 16, qs, qc, tail_p, head_p, tail, abort, limit_ns);
    }
  }
}

// The MMAs of one tile when its number of K chunks is known at compile time:
// for each chunk, wait for its stage, issue its four MMAs back to back and
// release the stage.  The tensor core's instruction queue is shallow: a few
// dozen instructions between two MMAs (descriptor arithmetic, a loop branch,
// a modulo) leave it idle, so descriptors advance by constants (start
// addresses in 16-byte units), the chunk loop is unrolled and the ring
// position wraps without a branch.  Returns false when a wait gave up.
template <int KCH, int OP>
__device__ __forceinline__ bool qk_mma_tile(uint32_t d_tmem, uint64_t da0, bool a_stream,
                                            uint64_t db0, uint32_t stage_units,
                                            uint32_t a_in_stage_units, bool extra, uint64_t dax,
                                            uint64_t dbx, uint32_t& stage, uint32_t& phase,
                                            uint32_t stages, uint64_t* full, uint64_t* empty,
                                            volatile int* abort, uint64_t wait_ns,
                                            uint32_t idesc) {
#pragma unroll
  for (int kc = 0; kc < KCH; ++kc) {
    if (!mbar_wait(&full[stage], phase, abort, wait_ns)) return false;
    tc_fence_after();
    const uint64_t db = db0 + (uint64_t)(stage * stage_units);
    const uint64_t da =
        a_stream ? db + a_in_stage_units : da0 + (uint64_t)(kc * (GT_ACHUNK >> 4));
    if (kc == 0 && extra) umma_f16_ss(d_tmem, dax, dbx, idesc, 0u);
#pragma unroll
    for (int kk = 0; kk < GT_KCH / 16; ++kk) {
      const uint32_t acc_in = (kc | kk) != 0 || extra;
      if constexpr (OP == 1)
        umma_i8_ss(d_tmem, da + 2 * kk, db + 2 * kk, idesc, acc_in);
      else
        umma_f16_ss(d_tmem, da + 2 * kk, db + 2 * kk, idesc, acc_in);
    }
    umma_commit(&empty[stage]);
    const uint32_t next = stage + 1;
    phase ^= next == stages ? 1u : 0u;
    stage = next == stages ? 0u : next;
  }
  return true;
}

template <int NPASS, int NBM, int KR, int OP, int MODE, int QD, int KCH = 0>
__global__ void __launch_bounds__(QK_THREADS, 1)
    knn_gemm_topk_queued_kernel(const __grid_constant__ CUtensorMap tm_a_hi,
                                const __grid_constant__ CUtensorMap tm_a_lo,
                                const __grid_constant__ CUtensorMap tm_b_hi,
                                const __grid_constant__ CUtensorMap tm_b_lo,
                                const __grid_constant__ CUtensorMap tm_b_x,
                                const KnnGemmParams p) {
  constexpr int NPA = NPASS == 1 ? 1 : 2;
  constexpr int QB = QK_QB;
  constexpr int CW = GT_BN / 2;   // columns per filter warp per tile
  constexpr int NCH = CW / 32;    // chunks of 32 columns (even)
  constexpr uint32_t IDESC = OP == 1 ? idesc_i8_s32(128, GT_BN) : idesc_f16_f32(128, GT_BN);
  static_assert(KR > 0 || MODE == 1, "the queued kernel keeps register lists");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const QueuedSmem lay = queued_smem(NPA, p.kchunks, p.stages, p.a_stream, p.extra, QD);
  uint8_t* a_res = smem + lay.a_off;
  uint8_t* ax = smem + lay.ax_off;
  uint8_t* stage_base = smem + lay.stage_off;
  uint8_t* x_ring = smem + lay.x_off;
  float4* qscore = reinterpret_cast<float4*>(smem + lay.q_off);
  int32_t* qcol = reinterpret_cast<int32_t*>(smem + lay.qcol_off);
  volatile uint32_t* qtail = reinterpret_cast<volatile uint32_t*>(smem + lay.qtail_off);
  volatile uint32_t* qhead = reinterpret_cast<volatile uint32_t*>(smem + lay.qhead_off);
  volatile unsigned long long* sthr =
      reinterpret_cast<volatile unsigned long long*>(smem + lay.thr_off);
  volatile unsigned long long* gthr =
      reinterpret_cast<volatile unsigned long long*>(smem + lay.gthr_off);
  uint32_t* unit_end = reinterpret_cast<uint32_t*>(smem + lay.misc_off);
  volatile uint32_t* units_done = unit_end + QK_END_RING;
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

  // every thread reads the same words, written by the prep kernels earlier
  // in the stream: the whole CTA returns, before any barrier or TMEM use
  if (p.skip_if != nullptr && (p.skip_if[0] | p.skip_if[2] | p.skip_if[4]) != 0u) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], QK_FILTER_WARPS);
    }
    *abort_flag = 0;
    for (int i = 0; i < QK_END_RING; ++i) unit_end[i] = 0u;
    *units_done = 0u;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < 2 * QB; i += blockDim.x) {
    qtail[i] = 0u;
    qhead[i] = 0u;
  }
  for (int i = threadIdx.x; i < QB; i += blockDim.x) {
    sthr[i] = 0ull;
    gthr[i] = 0ull;
  }
  if (warp == QK_MMA) {
    tmem_alloc(tmem_slot, 2 * GT_BN);
    tmem_relinquish();
    if (p.extra) {
      // the query-side half of the |b|^2 step: every row is
      // [-2^15, -2^11, -1, 0 ...], which against a base row's pieces
      // [x 2^7, y, z, 0 ...] of |b|^2 = x 2^22 + y 2^11 + z adds -|b|^2
      // (exactly: every product and partial sum is an integer < 2^31),
      // stored in the 32-byte swizzled layout (half c of row r at c ^ (r/4 % 2))
      const __half2 c01 = __floats2half2_rn(-32768.0f, -2048.0f);
      const __half2 c23 = __floats2half2_rn(-1.0f, 0.0f);
      uint4 data;
      data.x = *reinterpret_cast<const uint32_t*>(&c01);
      data.y = *reinterpret_cast<const uint32_t*>(&c23);
      data.z = 0u;
      data.w = 0u;
      for (int r = lane; r < 128; r += 32) {
        const int sw = (r >> 2) & 1;
        uint4* rowp = reinterpret_cast<uint4*>(ax + r * 32);
        rowp[sw] = data;
        rowp[sw ^ 1] = make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_shared();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == QK_PRODUCER) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      tma_prefetch_desc(&tm_a_hi);
      tma_prefetch_desc(&tm_b_hi);
      if (p.extra) tma_prefetch_desc(&tm_b_x);
      if (NPASS == 3) {
        tma_prefetch_desc(&tm_a_lo);
        tma_prefetch_desc(&tm_b_lo);
      }
      const uint32_t a_bytes = (uint32_t)(NPA * QB * 128);  // per K chunk
      uint32_t stage = 0, phase = 0, uidx = 0, tcount = 0;
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
        for (int t = t0; t < t1 && ok; ++t, ++tcount) {
          for (int kc = 0; kc < p.kchunks; ++kc) {
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.wait_ns)) {
              ok = false;
              break;
            }
            uint8_t* st = stage_base + (size_t)stage * lay.stage_bytes;
            const bool xk = p.extra && kc == 0;
            mbar_arrive_expect_tx(&full[stage], (uint32_t)(NPA * GT_BCHUNK) +
                                                    (p.a_stream ? a_bytes : 0u) +
                                                    (xk ? (uint32_t)GT_XCHUNK : 0u));
            const int brow = t * p.tile_stride * GT_BN;
            tma_load_2d(st, &tm_b_hi, &full[stage], kc * GT_KCH, brow);
            if (xk)
              tma_load_2d(x_ring + (size_t)(tcount % lay.x_slots) * GT_XCHUNK, &tm_b_x,
                          &full[stage], 0, brow);
            if (NPASS == 3)
              tma_load_2d(st + GT_BCHUNK, &tm_b_lo, &full[stage], kc * GT_KCH, brow);
            if (p.a_stream) {
              uint8_t* sa = st + NPA * GT_BCHUNK;
              tma_load_2d(sa, &tm_a_hi, &full[stage], kc * GT_KCH, qb * QB);
              if (NPASS == 3)
                tma_load_2d(sa + GT_ACHUNK, &tm_a_lo, &full[stage], kc * GT_KCH, qb * QB);
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
      // every load issued lands before the CTA may exit
      for (int s = 0; s < p.stages; ++s) {
        uint32_t par = ((uint32_t)s < stage) ? phase : (phase ^ 1);
        mbar_wait(&full[s], par, abort_flag, p.wait_ns);
      }
    }
  } else if (warp == QK_MMA) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, acc = 0, acc_ph = 0, uidx = 0, tcount = 0;
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
        if constexpr (KCH > 0) {
          // the lean form (the chunk count of this instantiation)
          const uint64_t da0 = sdesc_k128(smem_u32(a_res));
          const uint64_t db0 = sdesc_k128(smem_u32(stage_base));
          const uint64_t dax = sdesc_k32(smem_u32(ax));
          const uint64_t dbx0 = sdesc_k32(smem_u32(x_ring));
          uint32_t xs = lay.x_slots ? tcount % lay.x_slots : 0u;
          for (int t = t0; t < t1 && ok; ++t, ++tcount) {
            if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1, abort_flag, p.wait_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            ok = qk_mma_tile<KCH, OP>(
                tmem_base + acc * GT_BN, da0, p.a_stream != 0, db0, lay.stage_bytes >> 4,
                (uint32_t)(NPA * GT_BCHUNK) >> 4, p.extra != 0, dax,
                dbx0 + (uint64_t)(xs * (GT_XCHUNK >> 4)), stage, phase, (uint32_t)p.stages, full,
                empty, abort_flag, p.wait_ns, IDESC);
            if (!ok) break;
            umma_commit(&acc_full[acc]);
            acc ^= 1;
            acc_ph ^= acc == 0 ? 1u : 0u;
            const uint32_t xn = xs + 1;
            xs = xn == lay.x_slots ? 0u : xn;
          }
        } else
        for (int t = t0; t < t1 && ok; ++t, ++tcount) {
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
            if (p.extra && kc == 0)
              umma_f16_ss(d_tmem, sdesc_k32(smem_u32(ax)),
                          sdesc_k32(smem_u32(x_ring + (size_t)(tcount % lay.x_slots) * GT_XCHUNK)),
                          IDESC, 0u);
#pragma unroll
            for (int kk = 0; kk < GT_KCH / 16; ++kk) {
              const uint32_t acc_in = (kc | kk) != 0 || p.extra;
              if constexpr (OP == 1)
                umma_i8_ss(d_tmem, sdesc_k128(a_hi + kk * 32), sdesc_k128(b_hi + kk * 32), IDESC,
                           acc_in);
              else
                umma_f16_ss(d_tmem, sdesc_k128(a_hi + kk * 32), sdesc_k128(b_hi + kk * 32),
                            IDESC, acc_in);
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
  } else if (warp < QK_FILTER_WARPS) {
    // ------------------------------------------------------------- filter
    const int rg = warp & 3;         // TMEM lane quarter
    const int ch = warp >> 2;        // column half of the tile
    const int row = rg * 32 + lane;  // query within the block
    float4* qs = qscore + (size_t)ch * QD * 4 * QB + row;
    int32_t* qc = qcol + ch * QD * QB + row;
    volatile uint32_t* tail_p = qtail + ch * QB + row;
    volatile uint32_t* head_p = qhead + ch * QB + row;
    uint32_t tail = 0;
    uint32_t acc = 0, acc_ph = 0, uidx = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uidx) {
      const int qb = u % p.qblocks;
      const int split = u / p.qblocks;
      const int t0 = (int)((int64_t)split * p.tiles / p.splits);
      const int t1 = (int)((int64_t)(split + 1) * p.tiles / p.splits);
      const int64_t q = (int64_t)qb * QB + row;
      const bool q_ok = q < p.nq;
      const uint64_t tag = (uint64_t)(uidx + 1) << 32;
      const unsigned long long* gfl_q = p.gfloor + split * p.gfloor_split_stride + q;
      // padding rows offer nothing; the others start from the shared floor
      // (read once here; later rises arrive through shared memory)
      float thr = q_ok ? key_score(*reinterpret_cast<const volatile unsigned long long*>(gfl_q))
                       : INFINITY;
      for (int t = t0; t < t1 && ok; ++t) {
        if (MODE == 0 && q_ok) {
          // the select warp's floor of this unit and the other units' floor
          // as relayed (each a tile old at most)
          const unsigned long long x = sthr[row], g = gthr[row];
          if ((x & 0xFFFFFFFF00000000ull) == tag)
            thr = fmaxf(thr, __uint_as_float((uint32_t)x));
          if ((g & 0xFFFFFFFF00000000ull) == tag)
            thr = fmaxf(thr, __uint_as_float((uint32_t)g));
        }
        // one answer for the whole warp: the TMEM loads below are collective
        if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[acc], acc_ph, abort_flag, p.wait_ns))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr =
            tmem_base + ((uint32_t)(rg * 32) << 16) + acc * GT_BN + (uint32_t)(ch * CW);
        const int32_t col_base = (int32_t)((int64_t)t * p.tile_stride * GT_BN + ch * CW);
        // 64 columns per round trip to TMEM: two loads in flight, one wait
        // (a wait for each 32 columns would put four load latencies, not
        // two, on the path that frees the accumulator)
        uint32_t ra[32], rb[32];
        const float* nbt = p.nb + (int64_t)t * p.tile_stride * GT_BN + ch * CW;
#pragma unroll 1
        for (int c = 0; c < NCH; c += 2) {
          __syncwarp();
          tmem_ld32(taddr + c * 32, ra);
          tmem_ld32(taddr + (c + 1) * 32, rb);
          tmem_wait_ld_regs(ra);
          tmem_regs_ready(rb);
          if (c + 2 >= NCH) {
            // the accumulator is free once its last columns are in registers
            tc_fence_before();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
          }
          qk_filter32<NBM, OP, QD>(ra, nbt + c * 32, col_base + c * 32, thr, p.dot_offset, qs,
                                   qc, tail_p, head_p, tail, ok, abort_flag, p.wait_ns);
          qk_filter32<NBM, OP, QD>(rb, nbt + c * 32 + 32, col_base + c * 32 + 32, thr,
                                   p.dot_offset, qs, qc, tail_p, head_p, tail, ok, abort_flag,
                                   p.wait_ns);
        }
        ok = __all_sync(0xffffffffu, ok);
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
      }
      // the end of this unit for the query's select lane
      if (ok) ok = qk_push<QD>(nullptr, -1, qs, qc, tail_p, head_p, tail, abort_flag, p.wait_ns);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (!ok) {
      *abort_flag = 1;
      atomicOr(p.err, ERR_WAIT_EPILOGUE);
    }
  } else if (warp < QK_PRODUCER) {
    // ------------------------------------------------------------- select
    const int rg = warp - QK_FILTER_WARPS;
    const int row = rg * 32 + lane;
    // consumed chunks per column half's queue (two scalars: an array indexed
    // by the runtime half would live in local memory)
    uint32_t head0 = 0u, head1 = 0u;
    uint64_t key[KR > 0 ? KR : 1];
    uint32_t uidx = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uidx) {
      const int qb = u % p.qblocks;
      const int split = u / p.qblocks;
      const int64_t q = (int64_t)qb * QB + row;
      const bool q_ok = q < p.nq;
      const uint64_t tag = (uint64_t)(uidx + 1) << 32;
      unsigned long long* gfl_q = p.gfloor + split * p.gfloor_split_stride + q;
      const uint32_t self_id =
          (p.self_base >= 0 && q_ok) ? (uint32_t)(p.self_base + q) : 0xFFFFFFFFu;
      // MODE 0: start from the k best of the query block's latest finished
      // unit, so the list is full from its first chunk
      uint64_t floor = 0;
      if constexpr (MODE == 0) {
        const int ds = p.no_inherit ? 0 : *reinterpret_cast<volatile int*>(p.done + qb);
        __threadfence();
        const unsigned long long* src =
            reinterpret_cast<const unsigned long long*>(p.partial) +
            ((size_t)(ds > 0 ? ds - 1 : 0) * p.nq_pad + q) * p.k;
#pragma unroll
        for (int i = 0; i < KR; ++i) {
          uint64_t v = ~0ull;
          if (i < p.k) v = (ds > 0) ? __ldcg(src + i) : 0ull;
          key[i] = v;
        }
        floor = key[0];
      }
      {
        const uint64_t g = q_ok ? *reinterpret_cast<volatile unsigned long long*>(gfl_q) : 0ull;
        if (g > floor) floor = g;
      }
      float thr = key_score(floor);
      if (MODE == 0) sthr[row] = tag | __float_as_uint(thr);
      // collect mode: this unit's buffers and counts per column half
      uint64_t* cbuf0 = nullptr;
      uint64_t* cbuf1 = nullptr;
      int cnt0 = 0, cnt1 = 0;
      if (MODE == 1 && q_ok) {
        cbuf0 = p.collect + (((size_t)split * 2 + 0) * p.nq_pad + q) * (size_t)p.collect_cap;
        cbuf1 = p.collect + (((size_t)split * 2 + 1) * p.nq_pad + q) * (size_t)p.collect_cap;
      }
      uint32_t ended = 0;  // bit c: the end marker of column half c was seen
      long long idle_since = 0;
      uint32_t nap = QK_NAP_MIN_NS;  // idle poll interval, doubled while nothing arrives
      for (;;) {
        // each lane takes the next chunk of each of its query's two queues
        // (c static in the unrolled loop, so the per-half values stay in
        // registers)
        const uint64_t floor_before = floor;
        uint32_t mk[2] = {0u, 0u}, idb[2] = {0u, 0u}, en[2] = {0u, 0u};
        bool got = false;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint32_t hc = c ? head1 : head0;
          if (!((ended >> c) & 1u) && qk_ld_acquire(qtail + c * QB + row) != hc) {
            const uint32_t slot = hc % (uint32_t)QD;
            const int32_t col = qcol[(c * QD + slot) * QB + row];
            got = true;
            uint32_t mask = 0;
            if (col < 0) {
              ended |= 1u << c;
            } else {
              const float4* src = qscore + ((size_t)(c * QD + slot) * 4) * QB + row;
#pragma unroll
              for (int j4 = 0; j4 < 4; ++j4) {
                const float4 x = src[j4 * QB];
                mask |= (x.x >= thr ? 1u : 0u) << (4 * j4);
                mask |= (x.y >= thr ? 2u : 0u) << (4 * j4);
                mask |= (x.z >= thr ? 4u : 0u) << (4 * j4);
                mask |= (x.w >= thr ? 8u : 0u) << (4 * j4);
              }
              const int64_t valid = p.n_valid - (int64_t)col;
              if (valid < 16) mask &= valid <= 0 ? 0u : ((1u << valid) - 1u);
              idb[c] = (uint32_t)(p.id_offset + col);
              en[c] = c * QD + slot;
            }
            mk[c] = mask;
            if (mask == 0) {
              if (c) head1 = hc + 1u; else head0 = hc + 1u;
              qk_st_release(qhead + c * QB + row, hc + 1u);
            }
          }
        }
        // insert (or collect) the chunks' candidates: each round a lane
        // takes the next two marked scores (half 0's first), all lanes at
        // once; a chunk's slot is released once its last mark is taken
        while (__any_sync(0xffffffffu, (mk[0] | mk[1]) != 0u)) {
          uint64_t cand[2] = {0ull, 0ull};
#pragma unroll
          for (int t = 0; t < (MODE == 0 ? 2 : 1); ++t) {
            if (mk[0] | mk[1]) {
              const uint32_t h = mk[0] ? 0u : 1u;
              const uint32_t m = h ? mk[1] : mk[0];
              const int j = __ffs(m) - 1;
              const uint32_t rest = m & (m - 1);
              if (h) mk[1] = rest; else mk[0] = rest;
              const uint32_t e = h ? en[1] : en[0];
              const float vj = reinterpret_cast<const float*>(
                  qscore + ((size_t)e * 4 + (j >> 2)) * QB + row)[j & 3];
              const uint32_t id = (h ? idb[1] : idb[0]) + (uint32_t)j;
              const uint64_t x = make_key(vj, id);
              const bool take = x > floor && id != self_id;
              if constexpr (MODE == 1) {
                if (take) {
                  if (h == 0) {
                    if (cnt0 < p.collect_cap && cbuf0) cbuf0[cnt0] = x;
                    ++cnt0;
                  } else {
                    if (cnt1 < p.collect_cap && cbuf1) cbuf1[cnt1] = x;
                    ++cnt1;
                  }
                }
              } else {
                cand[t] = take ? x : 0ull;
              }
              if (rest == 0u) {
                const uint32_t nh = (h ? head1 : head0) + 1u;
                if (h) head1 = nh; else head0 = nh;
                qk_st_release(qhead + h * QB + row, nh);
              }
            }
          }
          if constexpr (MODE == 0) {
            const uint64_t hi = cand[0] > cand[1] ? cand[0] : cand[1];
            const uint64_t lo = cand[0] > cand[1] ? cand[1] : cand[0];
            if (hi != 0ull) {
              list_insert2<KR>(key, hi, lo);
              if (key[0] > floor) {
                floor = key[0];
                thr = key_score(floor);
              }
            }
          }
        }
        if (MODE == 0 && floor != floor_before) sthr[row] = tag | __float_as_uint(thr);
        if (__all_sync(0xffffffffu, ended == 3u)) break;
        if (!__any_sync(0xffffffffu, got)) {
          // nothing queued: pick up the other units' floor as relayed (its
          // score with the lowest id part: at or below their true floor)
          if (MODE == 0 && q_ok) {
            const unsigned long long g = gthr[row];
            if ((g & 0xFFFFFFFF00000000ull) == tag) {
              const uint64_t gk = (uint64_t)order_bits(__uint_as_float((uint32_t)g)) << 32;
              if (gk > floor) {
                floor = gk;
                thr = key_score(floor);
                sthr[row] = tag | __float_as_uint(thr);
              }
            }
          }
          const long long now = clock64();
          if (idle_since == 0) {
            idle_since = now;
          } else if (now - idle_since > qk_cycle_limit(p.wait_ns) || *abort_flag) {
            ok = false;
          }
          if (__any_sync(0xffffffffu, !ok)) {
            ok = false;
            break;
          }
          __nanosleep(nap);
          nap = nap * 2u < (uint32_t)QK_NAP_MAX_NS ? nap * 2u : (uint32_t)QK_NAP_MAX_NS;
        } else {
          idle_since = 0;
          nap = QK_NAP_MIN_NS;
        }
      }
      if (!ok) break;
      if constexpr (MODE == 1) {
        if (q_ok) {
          p.collect_count[((size_t)split * 2 + 0) * p.nq_pad + q] = cnt0;
          p.collect_count[((size_t)split * 2 + 1) * p.nq_pad + q] = cnt1;
        }
      } else {
        uint64_t* out = p.partial + ((size_t)split * p.nq_pad + q) * p.k;
#pragma unroll
        for (int i = 0; i < KR; ++i)
          if (i < p.k) out[i] = key[i];
        __threadfence();
        __syncwarp();
        // the last select warp to finish this unit marks the split finished
        if (lane == 0) {
          uint32_t* cnt = unit_end + uidx % QK_END_RING;
          if (atomicAdd(cnt, 1u) == QK_SELECT_WARPS - 1) {
            *cnt = 0u;
            __threadfence();
            atomicMax(p.done + qb, split + 1);
            atomicMax(const_cast<uint32_t*>(units_done), uidx + 1);
          }
        }
      }
    }
    if (!ok) {
      *abort_flag = 1;
      atomicOr(p.err, ERR_WAIT_EPILOGUE);
    }
  } else if (warp == QK_FLOORS && MODE == 0) {
    // ------------------------------------------------------------ relay
    // lane l serves rows l, l + 32, l + 64, l + 96 of the block: each round
    // publishes the list floors that rose (their scores, with the lowest id
    // part) and brings back the shared floor where it beats the list's
    uint32_t uidx = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x, ++uidx) {
      const int qb = u % p.qblocks;
      const int split = u / p.qblocks;
      const uint64_t tag = (uint64_t)(uidx + 1) << 32;
      unsigned long long* gfl[4];
      bool qk[4];
      uint64_t known[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int64_t q = (int64_t)qb * QB + lane + 32 * r;
        qk[r] = q < p.nq;
        gfl[r] = p.gfloor + split * p.gfloor_split_stride + q;
        known[r] = 0ull;
      }
      const long long start = clock64();
      while (*units_done <= uidx) {
        unsigned long long g[4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
          g[r] = qk[r] ? *reinterpret_cast<volatile unsigned long long*>(gfl[r]) : 0ull;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          if (!qk[r]) continue;
          const int row = lane + 32 * r;
          const unsigned long long x = sthr[row];
          if ((x & 0xFFFFFFFF00000000ull) == tag) {
            const uint64_t mine = (uint64_t)order_bits(__uint_as_float((uint32_t)x)) << 32;
            if (mine > known[r] && mine > g[r]) {
              atomicMax(gfl[r], (unsigned long long)mine);
              known[r] = mine;
            }
          }
          if (g[r] > known[r]) {
            known[r] = g[r];
            gthr[row] = tag | __float_as_uint(key_score(g[r]));
          }
        }
        if (*abort_flag || clock64() - start > qk_cycle_limit(p.wait_ns)) {
          ok = false;
          break;
        }
        __nanosleep(QK_RELAY_NAP_NS);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == QK_MMA) tmem_dealloc(tmem_base, 2 * GT_BN);
}

#endif  // __CUDACC__

}  // namespace mlxvs_b200
