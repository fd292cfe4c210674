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
};

#ifdef __CUDACC__

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__global__ void prep_rows_kernel(const PrepParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  uint32_t inexact = 0;
  float amax = 0.0f;
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
  }
  if (p.flags) {
    inexact = __any_sync(0xffffffffu, inexact);
    amax = warp_max(amax);
    if (lane == 0) {
      if (inexact) atomicOr(p.flags, 1u);
      atomicMax(p.flags + 1, __float_as_uint(amax));
    }
  }
}

// Vectorized prep for d % 4 == 0 and 16-byte aligned rows, one-pass only
// (lo == nullptr, cosine == 0): the benchmark's hot case.
__global__ void prep_rows_vec4_kernel(const PrepParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  uint32_t inexact = 0;
  float amax = 0.0f;
  const int d4 = p.d >> 2;
  const int dp4 = p.d_pad >> 2;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < p.n_pad;
       row += warps) {
    uint2* hrow = reinterpret_cast<uint2*>(p.hi + (size_t)row * p.d_pad);
    if (row >= p.n) {
      for (int c = lane; c < dp4; c += 32) hrow[c] = make_uint2(0u, 0u);
      if (p.norm_out && lane == 0) p.norm_out[row] = p.pad_norm;
      continue;
    }
    const float4* xr = reinterpret_cast<const float4*>(p.x + (size_t)row * p.d);
    float ss = 0.0f;
    for (int c = lane; c < dp4; c += 32) {
      float4 v = c < d4 ? __ldg(xr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      float w0 = v.x * p.mul, w1 = v.y * p.mul, w2 = v.z * p.mul, w3 = v.w * p.mul;
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(w0), fabsf(w1)), fmaxf(fabsf(w2), fabsf(w3))));
      w0 *= p.scale;
      w1 *= p.scale;
      w2 *= p.scale;
      w3 *= p.scale;
      __half2 h01 = __floats2half2_rn(w0, w1);
      __half2 h23 = __floats2half2_rn(w2, w3);
      float2 b01 = __half22float2(h01), b23 = __half22float2(h23);
      if (b01.x != w0 || b01.y != w1 || b23.x != w2 || b23.y != w3) inexact = 1;
      uint2 out;
      out.x = *reinterpret_cast<uint32_t*>(&h01);
      out.y = *reinterpret_cast<uint32_t*>(&h23);
      hrow[c] = out;
    }
    ss = warp_sum(ss);
    if (p.norm_out && lane == 0) p.norm_out[row] = p.norm_scale == 0.0f ? 0.0f : ss * p.norm_scale;
  }
  if (p.flags) {
    inexact = __any_sync(0xffffffffu, inexact);
    amax = warp_max(amax);
    if (lane == 0) {
      if (inexact) atomicOr(p.flags, 1u);
      atomicMax(p.flags + 1, __float_as_uint(amax));
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
// merge_keys: for each query, the best k of num_lists lists of k keys
// (list l, query q at lists[(l * list_rows + q) * k]), best first; then the
// output as keys and / or ids + distances of the given kind:
//   kind 1 (L2)      distance max(qq[q] - score, 0), +inf where missing
//                    (src/knn.cpp:122-131)
//   kind 0, 2        distance = score, -inf where missing
//   kind 3 (Hamming) distance = -score, +inf where missing
// One CTA per query: candidates are sorted in shared memory with a bitonic
// network, in rounds of MERGE_CAP - k new keys while more remain.
// ---------------------------------------------------------------------------
constexpr int MERGE_THREADS = 256;
constexpr int MERGE_CAP = 4096;

__global__ void __launch_bounds__(MERGE_THREADS)
    merge_keys_kernel(const uint64_t* __restrict__ lists, int32_t num_lists, int64_t list_rows,
                      int64_t nq, int32_t k, int32_t kind, const float* __restrict__ qq,
                      uint64_t* __restrict__ out_keys, int32_t* __restrict__ ids,
                      float* __restrict__ dist, int32_t cap) {
  extern __shared__ uint64_t buf[];  // [cap], a power of two > k
  const int64_t q = blockIdx.x;
  if (q >= nq) return;
  const int tid = threadIdx.x;
  const int64_t total = (int64_t)num_lists * k;
  int64_t next = 0;    // candidates consumed
  int kept = 0;        // valid sorted entries at the front of buf
  while (next < total || next == 0) {
    const int64_t room = cap - kept;
    const int64_t take = total - next < room ? total - next : room;
    int count = kept + (int)take;
    int size = 1;
    while (size < count) size <<= 1;
    if (size < 2) size = 2;
    for (int i = tid; i < size; i += MERGE_THREADS) {
      if (i >= kept) {
        int64_t c = next + (i - kept);
        uint64_t key = 0;
        if (i < count) {
          int64_t l = c / k, j = c - l * k;
          key = lists[((size_t)l * list_rows + q) * k + j];
        }
        buf[i] = key;
      }
    }
    __syncthreads();
    for (int s2 = 2; s2 <= size; s2 <<= 1) {
      for (int stride = s2 >> 1; stride > 0; stride >>= 1) {
        for (int i = tid; i < size; i += MERGE_THREADS) {
          int j = i ^ stride;
          if (j > i) {
            uint64_t a = buf[i], b = buf[j];
            bool desc = (i & s2) == 0;
            if (desc ? (a < b) : (a > b)) {
              buf[i] = b;
              buf[j] = a;
            }
          }
        }
        __syncthreads();
      }
    }
    next += take;
    kept = k < count ? k : count;
    if (next >= total) break;
  }
  float qn = (kind == 1 && qq) ? qq[q] : 0.0f;
  for (int j = tid; j < k; j += MERGE_THREADS) {
    uint64_t key = j < kept ? buf[j] : 0ull;
    if (out_keys) out_keys[(size_t)q * k + j] = key;
    if (ids) {
      int32_t id = key_id(key);
      ids[(size_t)q * k + j] = id;
      if (dist) {
        float s = key_score(key);
        float dv;
        if (kind == 1) {
          float dd = qn - s;
          dv = id >= 0 ? fmaxf(dd, 0.0f) : INFINITY;
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
