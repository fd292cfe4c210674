// Input conversion and list-merge kernels of the exact k-NN path.
#pragma once

#include "common.cuh"

namespace mlxvs_b200 {

// ---------------------------------------------------------------------------
// prep_rows: float32 rows [n, d] -> fp16 operand rows [n_pad, d_pad] laid
// out for the TMA (zero padded), one warp per row.
//
// The value converted is w = y * mul * scale, where y = x, or for cosine
// x / max(|x|, 1e-30) (the reference's unit_rows, src/knn.cpp:30-33), mul is
// 2 for L2 queries (the 2 q.b of src/knn.cpp:114, folded into the operand;
// exact) and scale a power of two.
//   lo == nullptr: hi = fp16(w); flags[0] |= 1 when some w is not exactly an
//                  fp16 (the exact one-pass path is then not taken).
//   lo != nullptr: hi = fp16(w), lo = fp16(w - hi): the split operands.
// flags[1] collects max |y * mul| as float bits (to choose the scale).
// norm_out[row] = sum(x^2) * norm_scale (float32; |b|^2 of src/knn.cpp:115
// or |q|^2 of :123), or 0 when norm_scale == 0; padding rows get pad_norm.
// xp (L2 base rows, may be null): |b|^2 as three fp16 pieces
// [x 2^7, y, z, 0 x 13] with |b|^2 = x 2^22 + y 2^11 + z, the operand of the
// GEMM's extra K step; fold_flag |= 1 when some |b|^2 is not an integer below
// 2^31 (then the pieces are unusable and the epilogue subtracts norm_out).
// ---------------------------------------------------------------------------
struct PrepParams {
  const float* x;
  int64_t n;
  int64_t n_pad;
  int32_t d;
  int32_t d_pad;
  int32_t cosine;
  float mul;
  float scale;
  __half* hi;
  __half* lo;
  float* norm_out;
  float norm_scale;
  float pad_norm;
  uint32_t* flags;
  __half* xp;
  uint32_t* fold_flag;
  // may be null: receives the largest sum(w^2) of a row (w before the
  // power-of-two scale), as float bits (for error bounds of fp16 scores)
  uint32_t* rownorm_max;
};

#ifdef __CUDACC__

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Lane 0 writes the 32-byte |b|^2 pieces of one row (zeros for padding rows).
__device__ __forceinline__ uint32_t write_pieces(__half* xp, int64_t row, float ss, bool valid) {
  uint4* dst = reinterpret_cast<uint4*>(xp + (size_t)row * 16);
  uint32_t bad = 0;
  uint4 lo = make_uint4(0u, 0u, 0u, 0u);
  if (valid) {
    if (!(ss == rintf(ss) && ss >= 0.0f && ss < 2147483648.0f)) {
      bad = 1;
    } else {
      const uint32_t u = (uint32_t)ss;
      const __half2 xy = __floats2half2_rn((float)((u >> 22) << 7), (float)((u >> 11) & 2047u));
      const __half2 z0 = __floats2half2_rn((float)(u & 2047u), 0.0f);
      lo.x = *reinterpret_cast<const uint32_t*>(&xy);
      lo.y = *reinterpret_cast<const uint32_t*>(&z0);
    }
  }
  dst[0] = lo;
  dst[1] = make_uint4(0u, 0u, 0u, 0u);
  return bad;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__global__ void prep_rows_kernel(const PrepParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  uint32_t inexact = 0, unfoldable = 0;
  float amax = 0.0f;
  float wmax = 0.0f;  // the largest sum(w^2) of this warp's rows
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < p.n_pad;
       row += warps) {
    __half* hrow = p.hi + (size_t)row * p.d_pad;
    __half* lrow = p.lo ? p.lo + (size_t)row * p.d_pad : nullptr;
    if (row >= p.n) {
      for (int c = lane; c < p.d_pad; c += 32) {
        hrow[c] = __float2half_rn(0.0f);
        if (lrow) lrow[c] = __float2half_rn(0.0f);
      }
      if (p.norm_out && lane == 0) p.norm_out[row] = p.pad_norm;
      if (p.xp && lane == 0) write_pieces(p.xp, row, 0.0f, false);
      continue;
    }
    const float* xr = p.x + (size_t)row * p.d;
    float ss = 0.0f;
    for (int c = lane; c < p.d; c += 32) {
      float v = __ldg(xr + c);
      ss += v * v;
    }
    ss = warp_sum(ss);
    float f = p.mul;
    if (p.cosine) {
      float den = fmaxf(sqrtf(ss), 1e-30f);
      // x / den as the reference divides; mul and scale are powers of two
      for (int c = lane; c < p.d_pad; c += 32) {
        float y = c < p.d ? __ldg(xr + c) / den : 0.0f;
        float w = y * f;
        amax = fmaxf(amax, fabsf(w));
        w *= p.scale;
        __half h = __float2half_rn(w);
        hrow[c] = h;
        if (lrow) {
          lrow[c] = __float2half_rn(w - __half2float(h));
        } else if (__half2float(h) != w) {
          inexact = 1;
        }
      }
    } else {
      for (int c = lane; c < p.d_pad; c += 32) {
        float w = c < p.d ? __ldg(xr + c) * f : 0.0f;
        amax = fmaxf(amax, fabsf(w));
        w *= p.scale;
        __half h = __float2half_rn(w);
        hrow[c] = h;
        if (lrow) {
          lrow[c] = __float2half_rn(w - __half2float(h));
        } else if (__half2float(h) != w) {
          inexact = 1;
        }
      }
    }
    if (p.norm_out && lane == 0) p.norm_out[row] = p.norm_scale == 0.0f ? 0.0f : ss * p.norm_scale;
    if (p.xp && lane == 0) unfoldable |= write_pieces(p.xp, row, ss, true);
    // sum(w^2) = mul^2 |x|^2 exactly (mul is a power of two); unit rows
    // (cosine) have norm at most 1 up to rounding, which the caller's
    // safety factor covers
    if (p.rownorm_max) wmax = fmaxf(wmax, p.cosine ? p.mul * p.mul : ss * p.mul * p.mul);
  }
  // one atomic per warp (a million rows on one address would serialize)
  if (p.rownorm_max && lane == 0) atomicMax(p.rownorm_max, __float_as_uint(wmax));
  if (p.fold_flag && __any_sync(0xffffffffu, unfoldable) && lane == 0) atomicOr(p.fold_flag, 1u);
  if (p.flags) {
    inexact = __any_sync(0xffffffffu, inexact);
    amax = warp_max(amax);
    if (lane == 0) {
      if (inexact) atomicOr(p.flags, 1u);
      atomicMax(p.flags + 1, __float_as_uint(amax));
    }
  }
}

// The same for d % 4 == 0 and 16-byte aligned rows, four values per lane
// and step (float4 loads, 8-byte half stores).  Cosine rows take one more
// pass over the row for the norm first.
// GENERAL = false compiles the plain case only (no cosine, no split plane):
// fewer registers, more rows in flight per SM.
template <bool GENERAL>
__global__ void prep_rows_vec4_kernel(const PrepParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  uint32_t inexact = 0, unfoldable = 0;
  float amax = 0.0f;
  float wmax = 0.0f;  // the largest sum(w^2) of this warp's rows
  const int d4 = p.d >> 2;
  const int dp4 = p.d_pad >> 2;
  const int64_t row0 = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  // plain case: each lane's first four values of the next row are loaded
  // one row ahead, so two loads per warp are in flight
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 ahead = (!GENERAL && row0 < p.n && lane < d4)
                     ? __ldg(reinterpret_cast<const float4*>(p.x + (size_t)row0 * p.d) + lane)
                     : zero4;
  for (int64_t row = row0; row < p.n_pad; row += warps) {
    const float4 first = ahead;
    if (!GENERAL) {
      const int64_t nr = row + warps;
      ahead = (nr < p.n && lane < d4)
                  ? __ldg(reinterpret_cast<const float4*>(p.x + (size_t)nr * p.d) + lane)
                  : zero4;
    }
    uint2* hrow = reinterpret_cast<uint2*>(p.hi + (size_t)row * p.d_pad);
    uint2* lrow = (GENERAL && p.lo) ? reinterpret_cast<uint2*>(p.lo + (size_t)row * p.d_pad) : nullptr;
    if (row >= p.n) {
      for (int c = lane; c < dp4; c += 32) {
        hrow[c] = make_uint2(0u, 0u);
        if (lrow) lrow[c] = make_uint2(0u, 0u);
      }
      if (p.norm_out && lane == 0) p.norm_out[row] = p.pad_norm;
      if (p.xp && lane == 0) write_pieces(p.xp, row, 0.0f, false);
      continue;
    }
    const float4* xr = reinterpret_cast<const float4*>(p.x + (size_t)row * p.d);
    float ss = 0.0f;
    float den = 1.0f;
    if (GENERAL && p.cosine) {
      for (int c = lane; c < d4; c += 32) {
        const float4 v = __ldg(xr + c);
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      ss = warp_sum(ss);
      den = fmaxf(sqrtf(ss), 1e-30f);
    }
    float ss_main = 0.0f;
    for (int c = lane; c < dp4; c += 32) {
      float4 v = (!GENERAL && c == lane) ? first : (c < d4 ? __ldg(xr + c) : zero4);
      if (GENERAL && p.cosine) {
        // x / den as the reference divides
        v.x = v.x / den;
        v.y = v.y / den;
        v.z = v.z / den;
        v.w = v.w / den;
      } else {
        ss_main += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      float w0 = v.x * p.mul, w1 = v.y * p.mul, w2 = v.z * p.mul, w3 = v.w * p.mul;
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(w0), fabsf(w1)), fmaxf(fabsf(w2), fabsf(w3))));
      w0 *= p.scale;
      w1 *= p.scale;
      w2 *= p.scale;
      w3 *= p.scale;
      __half2 h01 = __floats2half2_rn(w0, w1);
      __half2 h23 = __floats2half2_rn(w2, w3);
      const float2 b01 = __half22float2(h01), b23 = __half22float2(h23);
      uint2 out;
      out.x = *reinterpret_cast<uint32_t*>(&h01);
      out.y = *reinterpret_cast<uint32_t*>(&h23);
      hrow[c] = out;
      if (GENERAL && lrow) {
        __half2 l01 = __floats2half2_rn(w0 - b01.x, w1 - b01.y);
        __half2 l23 = __floats2half2_rn(w2 - b23.x, w3 - b23.y);
        uint2 lo;
        lo.x = *reinterpret_cast<uint32_t*>(&l01);
        lo.y = *reinterpret_cast<uint32_t*>(&l23);
        lrow[c] = lo;
      } else if (b01.x != w0 || b01.y != w1 || b23.x != w2 || b23.y != w3) {
        inexact = 1;
      }
    }
    if (!(GENERAL && p.cosine)) ss = warp_sum(ss_main);
    if (p.norm_out && lane == 0) p.norm_out[row] = p.norm_scale == 0.0f ? 0.0f : ss * p.norm_scale;
    if (p.xp && lane == 0) unfoldable |= write_pieces(p.xp, row, ss, true);
    // sum(w^2) = mul^2 |x|^2 exactly (mul is a power of two); unit rows
    // (cosine) have norm at most 1 up to rounding, which the caller's
    // safety factor covers
    if (p.rownorm_max) wmax = fmaxf(wmax, (GENERAL && p.cosine) ? p.mul * p.mul : ss * p.mul * p.mul);
  }
  // one atomic per warp (a million rows on one address would serialize)
  if (p.rownorm_max && lane == 0) atomicMax(p.rownorm_max, __float_as_uint(wmax));
  if (p.fold_flag && __any_sync(0xffffffffu, unfoldable) && lane == 0) atomicOr(p.fold_flag, 1u);
  if (p.flags) {
    inexact = __any_sync(0xffffffffu, inexact);
    amax = warp_max(amax);
    if (lane == 0) {
      if (inexact) atomicOr(p.flags, 1u);
      atomicMax(p.flags + 1, __float_as_uint(amax));
    }
  }
}

// The plain case (no cosine, no split plane) for rows of at most 128 values
// (d_pad <= 128): each warp converts four rows per step with its lanes' four
// float4 loads in flight together, then four interleaved warp sums.  Same
// outputs as prep_rows_vec4_kernel<false>, row for row.
__global__ void prep_rows4_kernel(const PrepParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  uint32_t inexact = 0, unfoldable = 0;
  float amax = 0.0f;
  float wmax = 0.0f;
  const int d4 = p.d >> 2;
  const int dp4 = p.d_pad >> 2;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  const int64_t warp_id = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (int64_t r0 = warp_id * 4; r0 < p.n_pad; r0 += warps * 4) {
    float4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t row = r0 + i;
      v[i] = (row < p.n && lane < d4)
                 ? __ldg(reinterpret_cast<const float4*>(p.x + (size_t)row * p.d) + lane)
                 : zero4;
    }
    float ss[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t row = r0 + i;
      float ss_main = 0.0f;
      ss_main += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
      ss[i] = ss_main;
      if (row < p.n_pad && lane < dp4) {
        float w0 = v[i].x * p.mul, w1 = v[i].y * p.mul, w2 = v[i].z * p.mul, w3 = v[i].w * p.mul;
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(w0), fabsf(w1)), fmaxf(fabsf(w2), fabsf(w3))));
        w0 *= p.scale;
        w1 *= p.scale;
        w2 *= p.scale;
        w3 *= p.scale;
        __half2 h01 = __floats2half2_rn(w0, w1);
        __half2 h23 = __floats2half2_rn(w2, w3);
        const float2 b01 = __half22float2(h01), b23 = __half22float2(h23);
        uint2 out;
        out.x = *reinterpret_cast<uint32_t*>(&h01);
        out.y = *reinterpret_cast<uint32_t*>(&h23);
        reinterpret_cast<uint2*>(p.hi + (size_t)row * p.d_pad)[lane] = out;
        if (b01.x != w0 || b01.y != w1 || b23.x != w2 || b23.y != w3) inexact = 1;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int i = 0; i < 4; ++i) ss[i] += __shfl_xor_sync(0xffffffffu, ss[i], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t row = r0 + i;
        if (row >= p.n_pad) break;
        if (row >= p.n) {
          if (p.norm_out) p.norm_out[row] = p.pad_norm;
          if (p.xp) write_pieces(p.xp, row, 0.0f, false);
          continue;
        }
        if (p.norm_out) p.norm_out[row] = p.norm_scale == 0.0f ? 0.0f : ss[i] * p.norm_scale;
        if (p.xp) unfoldable |= write_pieces(p.xp, row, ss[i], true);
        if (p.rownorm_max) wmax = fmaxf(wmax, ss[i] * p.mul * p.mul);
      }
    }
  }
  // the warps' flags and maxima meet in shared memory: one atomic per block
  // and word instead of one per warp (thousands on the same addresses)
  __shared__ float s_wmax[32], s_amax[32];
  __shared__ uint32_t s_bits[32];
  const int warp = threadIdx.x >> 5;
  inexact = __any_sync(0xffffffffu, inexact);
  unfoldable = __any_sync(0xffffffffu, unfoldable);
  amax = warp_max(amax);
  if (lane == 0) {
    s_wmax[warp] = wmax;
    s_amax[warp] = amax;
    s_bits[warp] = (inexact ? 1u : 0u) | (unfoldable ? 2u : 0u);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float bw = 0.0f, ba = 0.0f;
    uint32_t bits = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      bw = fmaxf(bw, s_wmax[w]);
      ba = fmaxf(ba, s_amax[w]);
      bits |= s_bits[w];
    }
    if (p.rownorm_max) atomicMax(p.rownorm_max, __float_as_uint(bw));
    if (p.fold_flag && (bits & 2u)) atomicOr(p.fold_flag, 1u);
    if (p.flags) {
      if (bits & 1u) atomicOr(p.flags, 1u);
      atomicMax(p.flags + 1, __float_as_uint(ba));
    }
  }
}

// |q|^2 per query in float32 (src/knn.cpp:123), one warp per row.
__global__ void row_sumsq_kernel(const float* x, int64_t n, int32_t d, float* out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < n;
       row += warps) {
    const float* xr = x + (size_t)row * d;
    float ss = 0.0f;
    for (int c = lane; c < d; c += 32) {
      float v = __ldg(xr + c);
      ss += v * v;
    }
    ss = warp_sum(ss);
    if (lane == 0) out[row] = ss;
  }
}

// ---------------------------------------------------------------------------
// merge_keys: for each query, the best k distinct keys of num_lists lists of
// k keys (list l, query q at lists[(l * list_rows + q) * k]), best first;
// scores are multiplied by `scale` (a power of two: the order is kept).
// Output as keys and / or ids + distances of the given kind:
//   kind 1 (L2)      distance max(qq[q] - score, 0), +inf where missing
//                    (src/knn.cpp:122-131)
//   kind 0, 2        distance = score, -inf where missing
//   kind 3 (Hamming) distance = -score, +inf where missing
// One CTA per query: candidates are sorted in shared memory with a bitonic
// network, in rounds of cap - k new keys while more remain; after each round
// warp 0 keeps the first k distinct keys (a key can sit in two lists when a
// unit started from another unit's list).
// ---------------------------------------------------------------------------
constexpr int MERGE_THREADS = 256;
constexpr int MERGE_CAP = 4096;

__global__ void __launch_bounds__(MERGE_THREADS)
    merge_keys_kernel(const uint64_t* __restrict__ lists, int32_t num_lists, int64_t list_rows,
                      int64_t nq, int32_t k, int32_t kind, const float* __restrict__ qq,
                      uint64_t* __restrict__ out_keys, int32_t* __restrict__ ids,
                      float* __restrict__ dist, int32_t cap, float scale) {
  extern __shared__ uint64_t buf[];  // [cap], a power of two > k
  __shared__ int kept_s;
  const int64_t q = blockIdx.x;
  if (q >= nq) return;
  const int tid = threadIdx.x;
  const int64_t total = (int64_t)num_lists * k;
  int64_t next = 0;  // candidates consumed
  int kept = 0;      // distinct sorted keys at the front of buf
  for (;;) {
    const int64_t room = cap - kept;
    const int64_t take = total - next < room ? total - next : room;
    const int count = kept + (int)take;
    int size = 2;
    while (size < count) size <<= 1;
    for (int i = tid; i < size; i += MERGE_THREADS) {
      if (i >= kept) {
        uint64_t key = 0;
        if (i < count) {
          const int64_t c = next + (i - kept);
          const int64_t l = c / k, j = c - l * k;
          key = lists[((size_t)l * list_rows + q) * k + j];
        }
        buf[i] = key;
      }
    }
    __syncthreads();
    for (int s2 = 2; s2 <= size; s2 <<= 1) {
      for (int stride = s2 >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < size; i += MERGE_THREADS) {
          const int j = i ^ stride;
          if (j > i) {
            const uint64_t a = buf[i], b = buf[j];
            const bool desc = (i & s2) == 0;
            if (desc ? (a < b) : (a > b)) {
              buf[i] = b;
              buf[j] = a;
            }
          }
        }
        __syncthreads();
      }
    }
    // compact the first k distinct non-empty keys to the front (in place:
    // an element moves only left, and only to where nothing is read later)
    if (tid < 32) {
      int w = 0;
      for (int base = 0; base < count && w < k; base += 32) {
        const int i = base + tid;
        const uint64_t key = i < count ? buf[i] : 0ull;
        const bool keep = key != 0 && (i == 0 || buf[i - 1] != key);
        const unsigned m = __ballot_sync(0xffffffffu, keep);
        __syncwarp();
        const int pos = w + __popc(m & ((1u << tid) - 1u));
        if (keep && pos < k) buf[pos] = key;
        __syncwarp();
        w += __popc(m);
      }
      if (tid == 0) kept_s = w < k ? w : k;
    }
    __syncthreads();
    kept = kept_s;
    next += take;
    if (next >= total) break;
  }
  const float qn = (kind == 1 && qq) ? qq[q] : 0.0f;
  for (int j = tid; j < k; j += MERGE_THREADS) {
    uint64_t key = j < kept ? buf[j] : 0ull;
    const float s = key_score(key) * scale;
    if (key != 0 && scale != 1.0f) key = make_key(s, ~(uint32_t)key);
    if (out_keys) out_keys[(size_t)q * k + j] = key;
    if (ids) {
      const int32_t id = key_id(key);
      ids[(size_t)q * k + j] = id;
      if (dist) {
        float dv;
        if (kind == 1) {
          dv = id >= 0 ? fmaxf(qn - s, 0.0f) : INFINITY;
        } else if (kind == 3) {
          dv = id >= 0 ? -s : INFINITY;
        } else {
          dv = id >= 0 ? s : -INFINITY;
        }
        dist[(size_t)q * k + j] = dv;
      }
    }
  }
}

// The same merge with one warp per query, for k <= 32 and at most 32 * MPL
// candidates: every lane holds up to MPL candidates in registers; each of the
// k rounds takes the warp's largest key (a shuffle max) and clears it from
// every lane (so a key present in two lists is taken once).
template <int MPL>
__global__ void __launch_bounds__(256)
    merge_keys_warp_kernel(const uint64_t* __restrict__ lists, int32_t num_lists,
                           int64_t list_rows, int64_t nq, int32_t k, int32_t kind,
                           const float* __restrict__ qq, uint64_t* __restrict__ out_keys,
                           int32_t* __restrict__ ids, float* __restrict__ dist, float scale) {
  const int lane = threadIdx.x & 31;
  const int64_t q = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (q >= nq) return;
  const int total = num_lists * k;
  uint64_t c[MPL];
#pragma unroll
  for (int m = 0; m < MPL; ++m) {
    const int idx = m * 32 + lane;
    uint64_t key = 0;
    if (idx < total) {
      const int l = idx / k, j = idx - l * k;
      key = __ldg(reinterpret_cast<const unsigned long long*>(lists) +
                  ((size_t)l * list_rows + q) * k + j);
    }
    c[m] = key;
  }
  const float qn = (kind == 1 && qq) ? qq[q] : 0.0f;
  for (int o = 0; o < k; ++o) {
    uint64_t best = c[0];
#pragma unroll
    for (int m = 1; m < MPL; ++m) best = c[m] > best ? c[m] : best;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, best, off);
      best = other > best ? other : best;
    }
#pragma unroll
    for (int m = 0; m < MPL; ++m)
      if (c[m] == best) c[m] = 0;
    if (lane == (o & 31)) {
      uint64_t key = best;
      const float sc = key_score(key) * scale;
      if (key != 0 && scale != 1.0f) key = make_key(sc, ~(uint32_t)key);
      if (out_keys) out_keys[(size_t)q * k + o] = key;
      if (ids) {
        const int32_t id = key_id(key);
        ids[(size_t)q * k + o] = id;
        if (dist) {
          float dv;
          if (kind == 1) {
            dv = id >= 0 ? fmaxf(qn - sc, 0.0f) : INFINITY;
          } else if (kind == 3) {
            dv = id >= 0 ? -sc : INFINITY;
          } else {
            dv = id >= 0 ? sc : -INFINITY;
          }
          dist[(size_t)q * k + o] = dv;
        }
      }
    }
  }
}

// At most this many candidates per query for merge_keys_quad_kernel (its
// 8 queries' lists fill 48 KB of shared memory).
constexpr int MERGE_QUAD_MAX = 768;

// Writes output slot o of query q: the key (scores times scale) and / or
// its id and distance of the given kind (see merge_keys).
__device__ __forceinline__ void merge_write(uint64_t key, int64_t q, int o, int k, int kind,
                                            float qn, float scale, uint64_t* out_keys,
                                            int32_t* ids, float* dist) {
  const float sc = key_score(key) * scale;
  if (key != 0 && scale != 1.0f) key = make_key(sc, ~(uint32_t)key);
  if (out_keys) out_keys[(size_t)q * k + o] = key;
  if (ids) {
    const int32_t id = key_id(key);
    ids[(size_t)q * k + o] = id;
    if (dist) {
      float dv;
      if (kind == 1) {
        dv = id >= 0 ? fmaxf(qn - sc, 0.0f) : INFINITY;
      } else if (kind == 3) {
        dv = id >= 0 ? -sc : INFINITY;
      } else {
        dv = id >= 0 ? sc : -INFINITY;
      }
      dist[(size_t)q * k + o] = dv;
    }
  }
}

// The lists of a merge whose lists live on different GPUs of the node (the
// row shards' keys, each in its GPU's exchange buffer, read over NVLink):
// list l is p[l] [nq][k].  failed holds the epoch of a step whose peer keys
// never arrived; that step's merge writes missing results instead of
// reading stale ones.
constexpr int MERGE_MAX_PEERS = 8;
struct PeerLists {
  const uint64_t* p[MERGE_MAX_PEERS];
  const volatile uint32_t* failed;
  uint32_t epoch;
};

__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* a) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}

// Whether merge_keys_quad_kernel takes a merge of num_lists lists of k keys.
__host__ __device__ inline bool merge_quad_fits(int64_t num_lists, int k) {
  return k <= 32 && num_lists <= 32 && num_lists * k <= MERGE_QUAD_MAX;
}

// The same merge with four lanes per query (eight queries per warp), for
// k <= KR <= 32, at most 32 lists and at most MERGE_QUAD_MAX candidates per
// query.  The warp copies its queries' rows of every list into shared
// memory (each list's rows are contiguous, so the copies are coalesced and
// all in flight at once).  Lane r of a query owns lists r, r + 4, ... .
// When every list of the warp is sorted, best first or best last, with
// empty slots (0) only at its worst end (the fused kernel's register lists
// are written worst first, merged lists best first), each of the k output
// slots is the best of the query's list heads (a max over a lane's heads,
// then over the four lanes by two shuffles), and every head equal to it
// moves on (a key present in two lists is taken once).  Otherwise the first
// lane of each query keeps its k best in a sorted register list
// (list_insert), skipping a key it already holds.  For L2 distances the
// kernel takes |q|^2 from qq, or computes it from queries [nq, d] when qq is
// null.
// With PEERS the lists are peers.p[l] (other GPUs' memory, read with
// system-scope loads, which no cache of this GPU answers from an older step).
template <int KR, bool PEERS = false>
__global__ void __launch_bounds__(32)
    merge_keys_quad_kernel(const uint64_t* __restrict__ lists, int32_t num_lists,
                           int64_t list_rows, int64_t nq, int32_t k, int32_t kind,
                           const float* __restrict__ qq, uint64_t* __restrict__ out_keys,
                           int32_t* __restrict__ ids, float* __restrict__ dist, float scale,
                           const float* __restrict__ queries, int32_t d,
                           const PeerLists peers = {}) {
  extern __shared__ __align__(16) uint64_t stage[];  // [num_lists][8][k]
  const int lane = threadIdx.x;
  const int64_t q0 = (int64_t)blockIdx.x * 8;
  const int rows = (int)(nq - q0 < 8 ? nq - q0 : 8);
  const int per_list = rows * k;
  bool lost = false;
  if constexpr (PEERS) lost = *peers.failed == peers.epoch;
  for (int l = 0; l < num_lists; ++l) {
    if constexpr (PEERS) {
      const uint64_t* src = peers.p[l] + (size_t)q0 * k;
      uint64_t* dst = stage + (size_t)l * 8 * k;
      for (int i = lane; i < per_list; i += 32) dst[i] = lost ? 0ull : ld_relaxed_sys(src + i);
    } else {
      const uint64_t* src = lists + ((size_t)l * list_rows + q0) * k;
      const uint32_t dst = (uint32_t)__cvta_generic_to_shared(stage + (size_t)l * 8 * k);
      for (int i = lane; i < per_list; i += 32)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(dst + 8u * (uint32_t)i),
                     "l"(src + i)
                     : "memory");
    }
  }
  // L2 without qq: |q|^2 of the warp's queries [nq, d] while the copies
  // land, in row_sumsq_kernel's order (lane-strided sums, then warp_sum)
  float qn_rows = 0.0f;
  if (kind == 1 && qq == nullptr && queries != nullptr) {
    float ssq[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) ssq[i] = 0.0f;
    for (int c = lane; c < d; c += 32) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < rows) {
          const float v = __ldg(queries + (size_t)(q0 + i) * d + c);
          ssq[i] += v * v;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float t = warp_sum(ssq[i]);
      if ((lane >> 2) == i) qn_rows = t;
    }
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
  __syncwarp();
  const int g = lane >> 2;  // query of the warp
  const int r = lane & 3;   // this lane's lists: r, r + 4, ...
  const bool row_ok = g < rows;
  const int64_t q = q0 + g;
  const uint64_t* mine = stage + (size_t)g * k;
  const size_t lstride = (size_t)8 * k;

  // which of this lane's lists run best last (bit i: list r + 4 i), and
  // whether every one is sorted
  uint32_t asc = 0;
  bool sorted = true;
  if (row_ok) {
    for (int i = 0, l = r; l < num_lists && sorted; ++i, l += 4) {
      const uint64_t* row = mine + l * lstride;
      bool up = true, down = true;
      uint64_t prev = row[0];
      for (int j = 1; j < k; ++j) {
        const uint64_t x = row[j];
        const bool both0 = x == 0 && prev == 0;
        up &= x > prev || both0;
        down &= x < prev || both0;
        prev = x;
      }
      if (up && !down) asc |= 1u << i;
      sorted = up || down;
    }
  }
  const float qn = (kind == 1 && row_ok) ? (qq ? qq[q] : qn_rows) : 0.0f;

  if (__all_sync(0xffffffffu, sorted)) {
    uint64_t head[8];
    int pos[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int l = r + 4 * i;
      pos[i] = ((asc >> i) & 1u) ? k - 1 : 0;
      head[i] = (row_ok && l < num_lists) ? mine[l * lstride + pos[i]] : 0ull;
    }
    for (int o = 0; o < k; ++o) {
      uint64_t best = head[0];
#pragma unroll
      for (int i = 1; i < 8; ++i) best = head[i] > best ? head[i] : best;
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        const uint64_t other = __shfl_xor_sync(0xffffffffu, best, off);
        best = other > best ? other : best;
      }
      if (r == 0 && row_ok) merge_write(best, q, o, k, kind, qn, scale, out_keys, ids, dist);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (best != 0 && head[i] == best) {
          const int l = r + 4 * i;
          pos[i] += ((asc >> i) & 1u) ? -1 : 1;
          head[i] = (pos[i] >= 0 && pos[i] < k) ? mine[l * lstride + pos[i]] : 0ull;
        }
      }
    }
    return;
  }

  if (r != 0 || !row_ok) return;
  // ascending: key[0] the worst kept (0 while fewer than k are held); slots
  // k .. KR-1 hold ~0 and never change
  uint64_t key[KR];
#pragma unroll
  for (int i = 0; i < KR; ++i) key[i] = i < k ? 0ull : ~0ull;
  for (int l = 0; l < num_lists; ++l) {
    const uint64_t* row = mine + l * lstride;
    for (int j = 0; j < k; ++j) {
      const uint64_t x = row[j];
      if (x <= key[0]) continue;
      bool held = false;
#pragma unroll
      for (int i = 0; i < KR; ++i) held |= i < k && key[i] == x;
      if (!held) list_insert<KR>(key, x);
    }
  }
#pragma unroll
  for (int i = 0; i < KR; ++i) {
    if (i >= k) break;
    merge_write(key[i], q, k - 1 - i, k, kind, qn, scale, out_keys, ids, dist);
  }
}

// The flags of one exchange step across the node's GPUs: this GPU's flag
// and every GPU's (peers' over NVLink), the step's epoch, and where a wait
// that gave up is recorded.
struct ExchangeFlags {
  volatile uint32_t* own;
  const volatile uint32_t* flag[MERGE_MAX_PEERS];
  int32_t world;
  uint32_t epoch;
  uint32_t* failed;
  uint32_t* err;
  long long limit_cycles;
};

// Publishes this GPU's keys of the epoch (written by the kernels before this
// one on the stream) and waits until every GPU has published its own: lane
// r polls GPU r's flag.  A wait that runs past the limit marks the step
// failed and raises ERR_WAIT_PEER instead of hanging.
__global__ void __launch_bounds__(32) exchange_wait_kernel(ExchangeFlags f) {
  const int lane = threadIdx.x;
  if (lane == 0) {
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f.own), "r"(f.epoch) : "memory");
  }
  __syncwarp();
  bool ok = true;
  if (lane < f.world) {
    const long long start = clock64();
    for (uint32_t i = 0;; ++i) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f.flag[lane]) : "memory");
      if ((int32_t)(v - f.epoch) >= 0) break;
      if ((i & 15u) == 15u && clock64() - start > f.limit_cycles) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  if (!__all_sync(0xffffffffu, ok) && lane == 0) {
    *f.failed = f.epoch;
    atomicOr(f.err, ERR_WAIT_PEER);
  }
}

// Outputs of a search over no rows: every id -1, every distance missing.
__global__ void fill_missing_kernel(int64_t count, int32_t kind, int32_t* ids, float* dist,
                                    uint64_t* keys) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (ids) ids[i] = -1;
    if (dist) dist[i] = (kind == 1 || kind == 3) ? INFINITY : -INFINITY;
    if (keys) keys[i] = 0ull;
  }
}

#endif  // __CUDACC__

}  // namespace mlxvs_b200
