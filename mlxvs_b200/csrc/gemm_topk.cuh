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
constexpr int GT_XCHUNK = GT_BN * 32;   // bytes of a tile's |b|^2 pieces (16 fp16 per row)
constexpr int GT_AX = 128 * 32;         // bytes of the constant query-side block
constexpr int GT_SHARE_TILES = 1;  // tiles between exchanges of the shared floor (power of 2)

struct KnnGemmParams {
  int32_t qblocks;   // query blocks of QB rows
  int32_t tiles;     // base tiles of GT_BN rows
  int32_t splits;    // base tile ranges per query block
  int32_t units;     // qblocks * splits
  int32_t kchunks;   // padded dimension / 64
  int32_t k;         // neighbors kept, <= heap capacity
  int32_t stages;    // depth of the base-chunk ring
  int32_t a_stream;  // 1: query chunks travel with the base chunks
  int32_t extra;     // 1: one more K=16 block per tile accumulates -|b|^2 (L2)
  int64_t n_valid;   // base rows
  int64_t nq;        // queries
  int64_t nq_pad;    // query rows of the partial lists (multiple of QB)
  int64_t id_offset;
  const float* nb;                 // [tiles * GT_BN]: subtracted from each dot
  uint64_t* partial;               // [splits][nq_pad][k] keys
  unsigned long long* gfloor;      // [nq_pad] shared floor keys (0 = none)
  int* done;                       // [qblocks] 1 + the latest split whose lists are written
  // OP 1 (Hamming on +-1 int8 codes): score = dot / 2 + dot_offset, with
  // dot_offset = -bits / 2, i.e. minus the Hamming distance
  float dot_offset;
  // base tile i of the units is tile i * tile_stride of the rows (1: all)
  int32_t tile_stride;
  // 0: a unit starts from the latest finished unit's lists of its query
  // block; 1: every unit starts empty (its list is its own rows' best)
  int32_t no_inherit;
  // the shared floors of split s are gfloor + s * gfloor_split_stride (0:
  // one floor per query for all units)
  int64_t gfloor_split_stride;
  // MODE 1 (collect): every candidate above the query's fixed floor that
  // column group c of the unit sees goes to collect[((split * CG + c) *
  // nq_pad + q) * collect_cap + i]; collect_count[(split * CG + c) * nq_pad +
  // q] receives how many there were (more than collect_cap means some were
  // dropped and the caller must search another way)
  uint64_t* collect;
  int32_t* collect_count;
  int32_t collect_cap;
  // >= 0: query q is the row with id self_base + q, which is never its own
  // neighbor (all_neighbors); -1: none
  int64_t self_base;
  uint32_t* err;                   // error word (bounded waits that gave up)
  uint64_t wait_ns;                // limit of every wait
  // non-null: a launch made before the host has read the prep's flags;
  // every CTA returns at entry when skip_if[0] | skip_if[2] | skip_if[4] is
  // non-zero (an operand is not exactly fp16, or |b|^2 cannot ride in the
  // MMA), and the host then runs the search the flags call for
  const uint32_t* skip_if;
};

// NBM = 0: the epilogue subtracts the per-row term nb from each dot (L2 when
// |b|^2 cannot ride in the MMA); NBM = 1: the accumulator already is the
// score (inner product, cosine, or L2 with the extra K block).
template <int QB, int NPASS, int CG>
struct GemmLayout {
  // CG column groups of 4 epilogue warps: warp w reads TMEM lane quarter
  // w % 4 (the hardware's rule) and column group w / 4 of each 256-column
  // accumulator; each (column group, query) keeps its own heap
  static constexpr int EW = 4 * CG;
  static constexpr int ROW_GROUPS = QB >= 32 ? QB / 32 : 1;
  static constexpr int ACTIVE_EW = CG * ROW_GROUPS;  // warps holding queries
  static constexpr int PRODUCER = EW;
  static constexpr int MMA = EW + 1;
  static constexpr int THREADS = (EW + 2) * 32;
  static constexpr int NPA = NPASS == 1 ? 1 : 2;  // operand planes: hi (, lo)
};

// Shared-memory offsets, computed identically on host and device.
struct GemmSmem {
  uint32_t a_off, a_bytes;      // resident query block (0 bytes when streamed)
  uint32_t ax_off;              // the constant query-side block of the extra K step
  uint32_t stage_off, stage_bytes;
  // heap mode: [k][CG * QB] keys, a heap per (column group, query); register
  // mode: [k][QB] keys, column group 1's list handed to group 0 at unit end
  uint32_t heap_off, heap_bytes;
  uint32_t sv_off;                // register mode: [4 * CG warps][16][32] floats, slow-path scores
  uint32_t nb_off;                // NBM 0: [4 * CG warps][256 / CG] floats, the tile's per-row terms
  uint32_t fl_off;                // [CG][QB] keys: each group's current floor, for its partners
  uint32_t bar_off;
  uint32_t total;
};

__host__ __device__ inline GemmSmem gemm_smem(int QB, int npa, int cg, int kchunks, int stages,
                                              int a_stream, int k, int extra, int kr, int nbm) {
  GemmSmem s;
  s.a_off = 0;
  s.a_bytes = a_stream ? 0u : (uint32_t)(npa * kchunks * GT_ACHUNK);
  s.ax_off = s.a_off + s.a_bytes;
  s.stage_off = s.ax_off + (extra ? (uint32_t)GT_AX : 0u);
  // stage: B hi [, B lo] [, A hi [, A lo]] [, |b|^2 pieces]
  s.stage_bytes = (uint32_t)(npa * (GT_BCHUNK + (a_stream ? GT_ACHUNK : 0)) +
                             (extra ? GT_XCHUNK : 0));
  s.heap_off = s.stage_off + (uint32_t)stages * s.stage_bytes;
  s.heap_bytes = (uint32_t)((kr ? 1 : cg) * QB * k * 8);
  s.sv_off = (s.heap_off + s.heap_bytes + 15u) & ~15u;
  s.nb_off = s.sv_off + (kr ? (uint32_t)(4 * cg) * 16u * 32u * 4u : 0u);
  s.fl_off = s.nb_off + (nbm == 0 ? 4u * GT_BN * 4u : 0u);
  s.bar_off = s.fl_off + (uint32_t)(cg * QB * 8);
  // full[stages], empty[stages], a_full, a_empty, acc_full[2], acc_empty[2], aux
  s.total = s.bar_off + (uint32_t)(2 * stages + 7) * 8u + 16u;
  return s;
}

#ifdef __CUDACC__

// Replaces the root of a min-heap of k keys (slot s at heap[s * HS]) by key,
// which is larger than the root.
template <int HS>
__device__ __forceinline__ void heap_replace_root(uint64_t* heap, int k, uint64_t key) {
  int i = 0;
  for (;;) {
    int l = 2 * i + 1;
    if (l >= k) break;
    uint64_t mv = heap[l * HS];
    int m = l;
    if (l + 1 < k) {
      uint64_t rv = heap[(l + 1) * HS];
      if (rv < mv) {
        mv = rv;
        m = l + 1;
      }
    }
    if (mv >= key) break;
    heap[i * HS] = mv;
    i = m;
  }
  heap[i * HS] = key;
}

struct EpiState {
  uint64_t* cbuf;  // MODE 1: this (query, column group)'s buffer of this unit
  int ccount;      // MODE 1: candidates offered to it so far
  uint32_t self_id;  // the query's own row id (all_neighbors), else 0xFFFFFFFF
  uint64_t floor;  // no candidate at or below this key can be in the result
  uint64_t gfl;    // the shared floor as last read or raised by this thread
  float thr;       // score of floor (-inf when none): the fast rejection test
};

// The slow path of 16 scores whose max reached the floor: each is offered
// to the heap in a rolled loop.  Out of line, with the scores and the state
// passed by value (registers), so the hot loop carries no call sites but one.
template <int HS>
__device__ __noinline__ EpiState epi_slow16(float v0, float v1, float v2, float v3, float v4,
                                            float v5, float v6, float v7, float v8, float v9,
                                            float v10, float v11, float v12, float v13,
                                            float v14, float v15, int64_t col0, int64_t n_valid,
                                            uint32_t id0, uint64_t* heap, int k, EpiState st) {
  const float v[16] = {v0, v1, v2, v3, v4, v5, v6, v7, v8, v9, v10, v11, v12, v13, v14, v15};
#pragma unroll 1
  for (int j = 0; j < 16; ++j) {
    const float vj = v[j];
    if (vj >= st.thr && col0 + j < n_valid) {
      const uint64_t key = make_key(vj, id0 + (uint32_t)j);
      if (key > st.floor && id0 + (uint32_t)j != st.self_id) {
        heap_replace_root<HS>(heap, k, key);
        const uint64_t root = heap[0];
        if (root > st.floor) st.floor = root;
        st.thr = key_score(st.floor);
      }
    }
  }
  return st;
}

// Waits on the register outputs of the preceding tcgen05.ld so the compiler
// cannot read them before the load has completed.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

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

// No instruction: ties the registers of a tcgen05.ld issued before the
// preceding tcgen05.wait::ld to this point, so that the compiler reads them
// only after that wait (which completes every load in flight).
__device__ __forceinline__ void tmem_regs_ready(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

__device__ __forceinline__ void sub2(float& a, float& b, float c, float d) {
  uint64_t x, y, z;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(c), "f"(d));
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(z) : "l"(x), "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(z));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// A sorted list of the KR best keys in registers, ascending: key[0] is the
// worst kept (0 while fewer than k are held); slots k .. KR-1 hold ~0 and
// never change.  Inserts x (x > key[0]) with a branch-free network: each
// slot takes its upper neighbour, x, or keeps its key.
template <int KR>
__device__ __forceinline__ void list_insert(uint64_t (&key)[KR], uint64_t x) {
  // b[i] = x beats key[i]; slot i then takes key[i + 1] when x also beats
  // that one, else x (one compare per slot, shared by its two neighbours)
  bool b[KR];
#pragma unroll
  for (int i = 0; i < KR; ++i) b[i] = x > key[i];
#pragma unroll
  for (int i = 0; i < KR; ++i) {
    const bool up = i + 1 < KR ? b[i + 1] : false;
    key[i] = up ? key[i + 1] : (b[i] ? x : key[i]);
  }
}

// Inserts two keys x >= y at once (y = 0: none) into the same list, keeping
// the KR best of the list and both.  In the merged ascending order y sits
// at #(keys < y) and x at #(keys < x) + 1; slot i of the result is the
// (i + 2)-th smallest of the union, so it takes key[i + 2] (both below it),
// y, key[i + 1] (only y below), x, or keeps key[i].
template <int KR>
__device__ __forceinline__ void list_insert2(uint64_t (&key)[KR], uint64_t x, uint64_t y) {
  bool bx[KR], by[KR];
#pragma unroll
  for (int i = 0; i < KR; ++i) {
    bx[i] = x > key[i];
    by[i] = y > key[i];
  }
  uint64_t n[KR];
#pragma unroll
  for (int i = 0; i < KR; ++i) {
    const bool by1 = i + 1 < KR ? by[i + 1] : false;
    const bool by2 = i + 2 < KR ? by[i + 2] : false;
    const bool bx1 = i + 1 < KR ? bx[i + 1] : false;
    const uint64_t k1 = i + 1 < KR ? key[i + 1] : 0ull;
    const uint64_t k2 = i + 2 < KR ? key[i + 2] : 0ull;
    n[i] = by1 ? (by2 ? k2 : y) : (bx[i] ? (bx1 ? k1 : x) : key[i]);
  }
#pragma unroll
  for (int i = 0; i < KR; ++i) key[i] = n[i];
}

// The register lists' slow path for 16 scores v[0..15] of columns col0..:
// every lane calls it (the votes are warp-wide); `mine` marks the lanes with
// a score at or above their floor.  Each such lane marks those scores in a
// 16-bit mask, the scores go through this warp's shared column (sv, stride
// 32), and the warp loops only while some lane still has marked scores
// (usually once or twice, not 16 times).
template <int KR, int MODE>
__device__ __forceinline__ void epi_slow_list16(const float* v, bool mine, int64_t col0,
                                                const KnnGemmParams& p,
                                                uint64_t (&key)[KR > 0 ? KR : 1], float* sv,
                                                EpiState& st) {
  if (!__any_sync(0xffffffffu, mine)) return;
  uint32_t mask = 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    sv[j * 32] = v[j];
    mask |= (v[j] >= st.thr ? 1u : 0u) << j;
  }
  if (!mine) mask = 0;
  if (col0 + 16 > p.n_valid) {
    const int64_t valid = p.n_valid - col0;
    mask &= valid <= 0 ? 0u : (valid >= 16 ? 0xFFFFu : ((1u << valid) - 1u));
  }
  __syncwarp();
  const uint32_t id0 = (uint32_t)(p.id_offset + col0);
  while (__any_sync(0xffffffffu, mask != 0)) {
    if (mask) {
      const int j = __ffs(mask) - 1;
      mask &= mask - 1;
      const float vj = sv[j * 32];
      const uint32_t id = id0 + (uint32_t)j;
      const uint64_t x = make_key(vj, id);
      if constexpr (MODE == 1) {
        // rows past nq (the last block's padding) have no buffer
        if (st.cbuf != nullptr && x > st.floor && id != st.self_id) {
          if (st.ccount < p.collect_cap) st.cbuf[st.ccount] = x;
          ++st.ccount;
        }
        continue;
      }
      if constexpr (KR > 0) {
        if (x > st.floor && id != st.self_id) {
          list_insert<KR>(key, x);
          if (key[0] > st.floor) st.floor = key[0];
          st.thr = key_score(st.floor);
        }
      }
    }
  }
  __syncwarp();
}

// 16 scores (raw dots r[o..o+15] minus the per-row terms nbs[0..15]): reject
// with one compare when their max is below the floor, else offer each.
template <int HS, int NBM, int KR, int OP, int MODE, int RN>
__device__ __forceinline__ void epi_sub16(const uint32_t (&r)[RN], int o, const float* nbs,
                                          int64_t col0, const KnnGemmParams& p, bool row_on,
                                          uint64_t* heap, uint64_t (&key)[KR > 0 ? KR : 1],
                                          float* sv, EpiState& st) {
  float v[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if constexpr (OP == 1)  // s32 dot of +-1 codes -> -(Hamming distance), exact
      v[j] = fmaf(__int2float_rn((int32_t)r[o + j]), 0.5f, p.dot_offset);
    else
      v[j] = __uint_as_float(r[o + j]);
  }
  if (NBM == 0) {
    const float4* nb4 = reinterpret_cast<const float4*>(nbs);
#pragma unroll
    for (int j4 = 0; j4 < 4; ++j4) {
      float4 t = nb4[j4];
      sub2(v[4 * j4 + 0], v[4 * j4 + 1], t.x, t.y);
      sub2(v[4 * j4 + 2], v[4 * j4 + 3], t.z, t.w);
    }
  }
  float m0 = max3(v[0], v[1], v[2]);
  float m1 = max3(v[3], v[4], v[5]);
  float m2 = max3(v[6], v[7], v[8]);
  float m3 = max3(v[9], v[10], v[11]);
  float m4 = max3(v[12], v[13], v[14]);
  float mx = max3(max3(m0, m1, m2), max3(m3, m4, v[15]), -INFINITY);
  if constexpr (KR == 0) {
    if (mx >= st.thr && row_on)
      st = epi_slow16<HS>(v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7], v[8], v[9], v[10],
                          v[11], v[12], v[13], v[14], v[15], col0, p.n_valid,
                          (uint32_t)(p.id_offset + col0), heap, p.k, st);
  } else {
    epi_slow_list16<KR, MODE>(v, row_on && mx >= st.thr, col0, p, key, sv, st);
  }
}

// 32 scores (r[0..31] minus nbs[0..31]) for the register lists: two
// 16-score maxima and one warp vote for both, so the common case (no lane
// above its floor) pays one vote and branch per 32 scores.  Used where the
// accumulator already is the score (NBM = 1; with the per-row terms the 32
// live scores spill) and for lists (in collect mode, where the floor is
// lower and votes succeed more often, it measured 1 % slower).  Config 1:
// -1.2 % kernel time.
template <int NBM, int KR, int OP, int MODE>
__device__ __forceinline__ void epi_sub32(const uint32_t (&r)[32], const float* nbs,
                                          int64_t col0, const KnnGemmParams& p, bool row_on,
                                          uint64_t (&key)[KR], float* sv, EpiState& st) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if constexpr (OP == 1)  // s32 dot of +-1 codes -> -(Hamming distance), exact
      v[j] = fmaf(__int2float_rn((int32_t)r[j]), 0.5f, p.dot_offset);
    else
      v[j] = __uint_as_float(r[j]);
  }
  if (NBM == 0) {
    const float4* nb4 = reinterpret_cast<const float4*>(nbs);
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4) {
      float4 t = nb4[j4];
      sub2(v[4 * j4 + 0], v[4 * j4 + 1], t.x, t.y);
      sub2(v[4 * j4 + 2], v[4 * j4 + 3], t.z, t.w);
    }
  }
  const float lo = max3(max3(max3(v[0], v[1], v[2]), max3(v[3], v[4], v[5]),
                             max3(v[6], v[7], v[8])),
                        max3(max3(v[9], v[10], v[11]), max3(v[12], v[13], v[14]), v[15]),
                        -INFINITY);
  const float hi = max3(max3(max3(v[16], v[17], v[18]), max3(v[19], v[20], v[21]),
                             max3(v[22], v[23], v[24])),
                        max3(max3(v[25], v[26], v[27]), max3(v[28], v[29], v[30]), v[31]),
                        -INFINITY);
  const bool a_lo = row_on && lo >= st.thr;
  if (__any_sync(0xffffffffu, a_lo || (row_on && hi >= st.thr))) {
    epi_slow_list16<KR, MODE>(v, a_lo, col0, p, key, sv, st);
    // the floor may have risen with the first half
    epi_slow_list16<KR, MODE>(v + 16, row_on && hi >= st.thr, col0 + 16, p, key, sv, st);
  }
}

template <int QB, int NPASS, int CG, int NBM, int KR, int OP = 0, int MODE = 0>
__global__ void __launch_bounds__(GemmLayout<QB, NPASS, CG>::THREADS, 1)
    knn_gemm_topk_kernel(const __grid_constant__ CUtensorMap tm_a_hi,
                         const __grid_constant__ CUtensorMap tm_a_lo,
                         const __grid_constant__ CUtensorMap tm_b_hi,
                         const __grid_constant__ CUtensorMap tm_b_lo,
                         const __grid_constant__ CUtensorMap tm_b_x, const KnnGemmParams p) {
  using L = GemmLayout<QB, NPASS, CG>;
  constexpr int NPA = L::NPA;
  constexpr int HS = CG * QB;     // heap slot stride
  constexpr int CW = GT_BN / CG;  // columns per epilogue warp per tile
  constexpr int NCH = CW / 32;    // chunks of 32 columns (even)
  constexpr uint32_t IDESC = OP == 1 ? idesc_i8_s32(128, GT_BN) : idesc_f16_f32(128, GT_BN);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const GemmSmem lay =
      gemm_smem(QB, NPA, CG, p.kchunks, p.stages, p.a_stream, p.k, p.extra, KR, NBM);
  uint8_t* a_res = smem + lay.a_off;
  uint8_t* ax = smem + lay.ax_off;
  // offset of the |b|^2 pieces inside a stage
  const uint32_t x_in_stage =
      (uint32_t)(NPA * (GT_BCHUNK + (p.a_stream ? GT_ACHUNK : 0)));
  uint8_t* stage_base = smem + lay.stage_off;
  uint64_t* heap_all = reinterpret_cast<uint64_t*>(smem + lay.heap_off);
  float* nb_all = reinterpret_cast<float*>(smem + lay.nb_off);
  float* sv_all = reinterpret_cast<float*>(smem + lay.sv_off);
  volatile unsigned long long* fl_all =
      reinterpret_cast<volatile unsigned long long*>(smem + lay.fl_off);
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
      mbar_init(&acc_empty[b], L::ACTIVE_EW);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < CG * QB; i += blockDim.x) fl_all[i] = 0ull;
  if (warp == L::MMA) {
    tmem_alloc(tmem_slot, 2 * GT_BN);
    tmem_relinquish();
    if (p.extra) {
      // the query-side half of the extra K step: every row is
      // [-2^15, -2^11, -1, 0 ...], which against a base row's pieces
      // [x 2^7, y, z, 0 ...] of |b|^2 = x 2^22 + y 2^11 + z adds -|b|^2
      // (exactly: every product and partial sum is an integer < 2^31).
      // Stored in the 32-byte swizzled layout: the 16-byte half c of row r
      // sits at half c ^ ((r >> 2) & 1).
      const __half2 c01 = __floats2half2_rn(-32768.0f, -2048.0f);
      const __half2 c23 = __floats2half2_rn(-1.0f, 0.0f);
      uint4 data;
      data.x = *reinterpret_cast<const uint32_t*>(&c01);
      data.y = *reinterpret_cast<const uint32_t*>(&c23);
      data.z = 0u;
      data.w = 0u;
      for (int r = lane; r < 128; r += 32) {
        const int sw = (r >> 2) & 1;
        uint4* row = reinterpret_cast<uint4*>(ax + r * 32);
        row[sw] = data;
        row[sw ^ 1] = make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_shared();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == L::PRODUCER) {
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
            const bool xk = p.extra && kc == 0;
            mbar_arrive_expect_tx(&full[stage], (uint32_t)(NPA * GT_BCHUNK) +
                                                    (p.a_stream ? a_bytes : 0u) +
                                                    (xk ? (uint32_t)GT_XCHUNK : 0u));
            const int brow = t * p.tile_stride * GT_BN;
            tma_load_2d(st, &tm_b_hi, &full[stage], kc * GT_KCH, brow);
            if (xk) tma_load_2d(st + x_in_stage, &tm_b_x, &full[stage], 0, brow);
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
      // Every load issued lands before the CTA may exit: the last arm of each
      // stage completes by itself (bounded wait all the same).
      for (int s = 0; s < p.stages; ++s) {
        uint32_t par = ((uint32_t)s < stage) ? phase : (phase ^ 1);
        mbar_wait(&full[s], par, abort_flag, p.wait_ns);
      }
    }
  } else if (warp == L::MMA) {
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
            if (p.extra && kc == 0)
              umma_f16_ss(d_tmem, sdesc_k32(smem_u32(ax)), sdesc_k32(b_hi + x_in_stage), IDESC,
                          0u);
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
  } else if (warp < L::EW && (warp & 3) < L::ROW_GROUPS) {
    // ------------------------------------------------------------- epilogue
    const int rg = warp & 3;          // TMEM lane quarter
    const int ch = warp >> 2;         // column group of the tile
    const int row = rg * 32 + lane;   // query within the block
    // with QB < 32 the lanes past QB only join the warp-collective loads
    const bool row_on = row < QB;
    uint64_t* heap = heap_all + ch * QB + (row_on ? row : 0);
    float* nbw = nb_all + warp * CW;  // this warp's per-row terms of the tile
    float* sv = sv_all + warp * 512 + lane;
    uint64_t key[KR > 0 ? KR : 1];    // register mode: the sorted list
    uint32_t acc = 0, acc_ph = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.units && ok; u += gridDim.x) {
      const int qb = u % p.qblocks;
      const int split = u / p.qblocks;
      const int t0 = (int)((int64_t)split * p.tiles / p.splits);
      const int t1 = (int)((int64_t)(split + 1) * p.tiles / p.splits);
      const int64_t q = (int64_t)qb * QB + row;
      const bool q_ok = row_on && q < p.nq;
      // Start from the k best of the query block's latest finished unit (a
      // min-heap as written): the heap is full from its first tile, so its
      // root is a real floor and every improvement reaches the shared floor.
      // Column group 1 only takes the floor (its heap would duplicate them).
      const int ds =
          (MODE == 1 || p.no_inherit) ? 0 : *reinterpret_cast<volatile int*>(p.done + qb);
      __threadfence();
      uint64_t inherited = 0;
      if constexpr (KR > 0) {
        const unsigned long long* src =
            reinterpret_cast<const unsigned long long*>(p.partial) +
            ((size_t)(ds > 0 ? ds - 1 : 0) * p.nq_pad + q) * p.k;
#pragma unroll
        for (int i = 0; i < KR; ++i) {
          uint64_t v = ~0ull;
          if (i < p.k) v = (row_on && ds > 0 && ch == 0) ? __ldcg(src + i) : 0ull;
          key[i] = v;
        }
        if (row_on && ds > 0) inherited = __ldcg(src);
      } else if (row_on) {
        if (ds > 0) {
          const uint64_t* src = p.partial + ((size_t)(ds - 1) * p.nq_pad + q) * p.k;
          for (int s = 0; s < p.k; ++s) {
            const uint64_t key = __ldcg(reinterpret_cast<const unsigned long long*>(src) + s);
            if (ch == 0) heap[s * HS] = key;
          }
          inherited = __ldcg(reinterpret_cast<const unsigned long long*>(src));
        } else if (ch == 0) {
          for (int s = 0; s < p.k; ++s) heap[s * HS] = 0;
        }
        if (ch == 1)
          for (int s = 0; s < p.k; ++s) heap[s * HS] = 0;
      }
      EpiState st;
      st.self_id = (p.self_base >= 0 && q_ok) ? (uint32_t)(p.self_base + q) : 0xFFFFFFFFu;
      unsigned long long* gfl_q = p.gfloor + split * p.gfloor_split_stride + q;
      st.cbuf = (MODE == 1 && q_ok)
                    ? p.collect + (((size_t)split * CG + ch) * p.nq_pad + q) * (size_t)p.collect_cap
                    : nullptr;
      st.ccount = 0;
      st.gfl = q_ok ? *reinterpret_cast<volatile unsigned long long*>(gfl_q) : 0ull;
      if (inherited > st.gfl) st.gfl = inherited;
      st.floor = st.gfl;
      st.thr = key_score(st.floor);
      if (MODE == 1 && !q_ok) st.thr = INFINITY;  // padding rows collect nothing
      uint64_t gnext = st.gfl;
      float4 nbr[CW / 128];
      if (NBM == 0 && t0 < t1) {
#pragma unroll
        for (int i = 0; i < CW / 128; ++i)
          nbr[i] = __ldg(reinterpret_cast<const float4*>(
                             p.nb + (int64_t)t0 * p.tile_stride * GT_BN + ch * CW) +
                         lane + 32 * i);
      }
      for (int t = t0; t < t1; ++t) {
        // stage this tile's per-row terms, prefetch the next tile's
        if (NBM == 0) {
          __syncwarp();
#pragma unroll
          for (int i = 0; i < CW / 128; ++i)
            reinterpret_cast<float4*>(nbw)[lane + 32 * i] = nbr[i];
          __syncwarp();
        }
        if (NBM == 0 && t + 1 < t1) {
#pragma unroll
          for (int i = 0; i < CW / 128; ++i)
            nbr[i] = __ldg(
                reinterpret_cast<const float4*>(
                    p.nb + (int64_t)(t + 1) * p.tile_stride * GT_BN + ch * CW) +
                lane + 32 * i);
        }
        if (!mbar_wait(&acc_full[acc], acc_ph, abort_flag, p.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr =
            tmem_base + ((uint32_t)(rg * 32) << 16) + acc * GT_BN + (uint32_t)(ch * CW);
        const int64_t col_base = (int64_t)t * p.tile_stride * GT_BN + ch * CW;
        if constexpr (KR >= 32) {
          // the long register lists leave room for 16-column loads only
          uint32_t ra[16], rb[16];
          tmem_ld16(taddr, ra);
          tmem_wait_ld_regs(ra);
#pragma unroll 1
          for (int c = 0; c < 2 * NCH; c += 2) {
            __syncwarp();
            tmem_ld16(taddr + (c + 1) * 16, rb);
            epi_sub16<HS, NBM, KR, OP, MODE>(ra, 0, nbw + c * 16, col_base + c * 16, p, row_on, heap, key, sv, st);
            __syncwarp();
            tmem_wait_ld_regs(rb);
            if (c + 2 < 2 * NCH) {
              tmem_ld16(taddr + (c + 2) * 16, ra);
            } else {
              tc_fence_before();
              if (lane == 0) mbar_arrive(&acc_empty[acc]);
            }
            epi_sub16<HS, NBM, KR, OP, MODE>(rb, 0, nbw + c * 16 + 16, col_base + c * 16 + 16, p, row_on, heap, key, sv, st);
            if (c + 2 < 2 * NCH) {
              __syncwarp();
              tmem_wait_ld_regs(ra);
            }
          }
        } else {
        // 64 columns per round trip to TMEM: two loads in flight, one wait
        uint32_t ra[32], rb[32];
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
          if constexpr (KR > 0 && NBM == 1 && MODE == 0) {
            epi_sub32<NBM, KR, OP, MODE>(ra, nbw + c * 32, col_base + c * 32, p, row_on, key, sv, st);
            epi_sub32<NBM, KR, OP, MODE>(rb, nbw + c * 32 + 32, col_base + c * 32 + 32, p, row_on, key, sv, st);
          } else {
            epi_sub16<HS, NBM, KR, OP, MODE>(ra, 0, nbw + c * 32, col_base + c * 32, p, row_on, heap, key, sv, st);
            epi_sub16<HS, NBM, KR, OP, MODE>(ra, 16, nbw + c * 32 + 16, col_base + c * 32 + 16, p, row_on, heap, key, sv, st);
            epi_sub16<HS, NBM, KR, OP, MODE>(rb, 0, nbw + c * 32 + 32, col_base + c * 32 + 32, p, row_on, heap, key, sv, st);
            epi_sub16<HS, NBM, KR, OP, MODE>(rb, 16, nbw + c * 32 + 48, col_base + c * 32 + 48, p, row_on, heap, key, sv, st);
          }
        }
        }
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1;
        if (CG == 2 && row_on && MODE == 0) {
          // the other column group's floor for this query (a tile old at most)
          const uint64_t mine = KR > 0 ? key[0] : heap[0];
          fl_all[ch * QB + row] = mine;
          const uint64_t theirs = fl_all[(ch ^ 1) * QB + row];
          if (theirs > st.floor) {
            st.floor = theirs;
            st.thr = key_score(theirs);
          }
        }
        if (q_ok && ((t - t0) & (GT_SHARE_TILES - 1)) == GT_SHARE_TILES - 1) {
          // the shared floor loaded one tile ago (its latency is hidden
          // behind this tile's work); then publish the best floor this
          // thread knows if it beats the last shared one seen, and load the
          // shared one for the next tile
          const uint64_t g = gnext;
          if (g > st.gfl) {
            st.gfl = g;
            if (g > st.floor) {
              st.floor = g;
              st.thr = key_score(g);
            }
          }
          if (st.floor > st.gfl) {
            atomicMax(gfl_q, (unsigned long long)st.floor);
            st.gfl = st.floor;
          }
          gnext = *reinterpret_cast<volatile unsigned long long*>(gfl_q);
        }
      }
      if (!ok) break;
      if constexpr (MODE == 1) {
        // each column group's count of its own buffer
        if (q_ok) p.collect_count[((size_t)split * CG + ch) * p.nq_pad + q] = st.ccount;
        continue;
      }
      if (CG == 2) {
        // the two column groups of each query meet: group 1's keys go into
        // group 0's selection, which is written out as the unit's list
        if constexpr (KR > 0) {
          if (ch == 1 && row_on) {
#pragma unroll
            for (int i = 0; i < KR; ++i)
              if (i < p.k) heap_all[i * QB + row] = key[i];
          }
        }
        asm volatile("bar.sync %0, 64;" ::"r"(1 + rg) : "memory");
        if (ch == 0 && row_on) {
          if constexpr (KR > 0) {
#pragma unroll 1
            for (int i = 0; i < p.k; ++i) {
              const uint64_t x = heap_all[i * QB + row];
              if (x > key[0]) list_insert<KR>(key, x);
            }
          } else {
            const uint64_t* other = heap + QB;
            for (int s = 0; s < p.k; ++s) {
              const uint64_t kx = other[s * HS];
              if (kx > heap[0]) heap_replace_root<HS>(heap, p.k, kx);
            }
          }
        }
      }
      if (ch == 0) {
        if (row_on) {
          uint64_t* out = p.partial + ((size_t)split * p.nq_pad + q) * p.k;
          if constexpr (KR > 0) {
#pragma unroll
            for (int i = 0; i < KR; ++i)
              if (i < p.k) out[i] = key[i];
          } else {
            for (int s = 0; s < p.k; ++s) out[s] = heap[s * HS];
          }
          __threadfence();
        }
        // all of group 0's lists are out: mark the split finished
        asm volatile("bar.sync %0, %1;" ::"r"(5), "r"(L::ROW_GROUPS * 32) : "memory");
        if (warp == 0 && lane == 0) atomicMax(p.done + qb, split + 1);
      }
      if (CG == 2) {
        // floors are per query: clear this one before the partner can start
        // the next unit and read it
        if (row_on) fl_all[ch * QB + row] = 0ull;
        asm volatile("bar.sync %0, 64;" ::"r"(1 + rg) : "memory");
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
  if (warp == L::MMA) tmem_dealloc(tmem_base, 2 * GT_BN);
}

#endif  // __CUDACC__

}  // namespace mlxvs_b200
