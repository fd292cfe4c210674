// Device helpers shared by the k-NN kernels: 64-bit (score, id) keys, bounded
// mbarrier waits, TMA (cp.async.bulk.tensor) loads and tcgen05 (5th-gen
// tensor core + tensor memory) wrappers, all as inline PTX for sm_100a.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mlxvs_b200 {

// ---------------------------------------------------------------------------
// Keys.  A candidate (score s, id i) is the 64-bit key
//   (order_bits(s) << 32) | (uint32)~i
// so that a larger key is a better candidate: higher score first, then lower
// id as an unsigned number (the reference's mlxvs_before, src/kernels.h:20-23,
// whose selection uses the same order_bits map, src/kernels.h:16-19).
// Key 0 is an empty slot: every real candidate has a larger key.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t order_bits(float v) {
#ifdef __CUDA_ARCH__
  uint32_t u = __float_as_uint(v);
#else
  uint32_t u;
  memcpy(&u, &v, 4);
#endif
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__host__ __device__ __forceinline__ float from_order_bits(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k ^ 0x80000000u) : ~k;
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float v;
  memcpy(&v, &u, 4);
  return v;
#endif
}

__host__ __device__ __forceinline__ uint64_t make_key(float s, uint32_t id) {
  return ((uint64_t)order_bits(s) << 32) | (uint64_t)(~id);
}

__host__ __device__ __forceinline__ float key_score(uint64_t key) {
  return key == 0 ? -INFINITY : from_order_bits((uint32_t)(key >> 32));
}

__host__ __device__ __forceinline__ int32_t key_id(uint64_t key) {
  return key == 0 ? -1 : (int32_t)(~(uint32_t)key);
}

// Error word written by kernels whose bounded waits gave up.
enum : uint32_t {
  ERR_WAIT_PRODUCER = 1u,
  ERR_WAIT_MMA = 2u,
  ERR_WAIT_EPILOGUE = 4u,
  ERR_WAIT_PEER = 8u,
};

#ifdef __CUDACC__

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// A time limit in SM cycles for a limit in nanoseconds: 2 cycles per
// nanosecond lasts at least as long at any clock up to 2 GHz.  Waits count
// cycles with clock64 (a register read) rather than reading %globaltimer,
// which takes on the order of a microsecond: a waiting thread that reads it
// when its barrier is not yet complete would notice the completion that
// much later.
__device__ __forceinline__ long long wait_cycles(uint64_t limit_ns) {
  return (long long)(2 * limit_ns);
}

// Waits for the phase of the given parity to complete, for at most about
// limit_ns (checked every 256 polls).  Returns false when it gave up, or when
// *abort was raised by another role of the CTA.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*abort) return false;
      if (clock64() - start > wait_cycles(limit_ns)) return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA: tiled 2-D load global -> shared, completion counted on an mbarrier.
// x is the innermost (contiguous) coordinate in elements; x * element size
// must be a multiple of 16 bytes (all callers use multiples of 64 fp16).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Untiled bulk copy global -> shared (both 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory allocation, MMA issue, commit, loads.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, fp16 inputs, fp32 accumulators.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same with signed 8-bit operands and signed 32-bit accumulators
// (kind::i8; K = 32 bytes per instruction, the same smem stepping as f16).
__device__ __forceinline__ void umma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on bar when every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane (32x32b shape:
// warp w reads lanes 32*(w%4) .. +31).
// 16 consecutive fp32 columns of this warp's 32 TMEM lanes (one row per
// thread); completes at the next tcgen05.wait::ld.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15},"
      " [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31},"
      " [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored in the
// 128-byte swizzled layout that TMA writes with CU_TENSOR_MAP_SWIZZLE_128B:
// rows of 128 bytes (64 fp16), 8-row atoms of 1024 bytes (the stride byte
// offset), tile start 1024-byte aligned.  Advancing K by 16 fp16 inside the
// atom adds 32 bytes to the start address.
__device__ __forceinline__ uint64_t sdesc_k128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address, 16-byte units
  d |= (uint64_t)1 << 16;                    // leading byte offset (unused here)
  d |= (uint64_t)(1024 >> 4) << 32;          // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                    // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                    // swizzle mode: 128-byte
  return d;
}

// The same for a K-major tile of 16 fp16 per row in the 32-byte swizzled
// layout (CU_TENSOR_MAP_SWIZZLE_32B): 32-byte rows, 8-row atoms of 256 bytes,
// tile start 256-byte aligned; one K=16 step covers the whole row.
__device__ __forceinline__ uint64_t sdesc_k32(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address, 16-byte units
  d |= (uint64_t)1 << 16;                    // leading byte offset (unused here)
  d |= (uint64_t)(256 >> 4) << 32;           // stride byte offset: 8 rows x 32 B
  d |= (uint64_t)1 << 46;                    // descriptor version (sm_100)
  d |= (uint64_t)6 << 61;                    // swizzle mode: 32-byte
  return d;
}

// Instruction descriptor of kind::f16: fp16 A and B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4)                       // D format: f32
         | (0u << 7) | (0u << 10)        // A, B format: f16
         | (0u << 15) | (0u << 16)       // A, B K-major
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | ((uint32_t)(M >> 4) << 24);   // M / 16
}

// Instruction descriptor of kind::i8: signed 8-bit A and B (K-major), s32
// accumulators, M x N.
__host__ __device__ constexpr uint32_t idesc_i8_s32(int M, int N) {
  return (2u << 4)                       // D format: s32
         | (1u << 7) | (1u << 10)        // A, B format: signed 8-bit
         | (0u << 15) | (0u << 16)       // A, B K-major
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | ((uint32_t)(M >> 4) << 24);   // M / 16
}

#endif  // __CUDACC__

}  // namespace mlxvs_b200
