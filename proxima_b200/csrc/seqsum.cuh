// seqsum.cuh — the left-to-right f64 sum of non-negative f32 values, computed
// in parallel and equal bit for bit to the sequential loop
//     s = 0.0; for v in values { s += f64::from(v) }
// that the reference uses for k-means inertia and the k-means++ total and
// cumulative search (crates/proxima-quantize/src/kmeans.rs:89-91,162-177).
//
// Method. Every value is converted to a 128-bit fixed-point integer with a
// common least-significant-bit weight 2^L chosen from the largest value, so
// that n values cannot overflow. Prefix sums of integers are exact in any
// order. If every prefix P_i is exactly representable as an f64 (at most 53
// significant bits), the sequential loop never rounds and its partial sums are
// exactly P_i: s_i = P_i. The first index at which that fails (a prefix needing
// more than 53 bits, or a value finer than 2^L) is found with an atomic min;
// from there on the sum continues sequentially in one thread, in f64, exactly
// like the reference loop. Data whose distances are well above the rounding
// grain (the usual case) never takes that tail.
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace pxc {
namespace seqsum {

typedef unsigned __int128 u128;

constexpr int THREADS = 256;
constexpr int ITEMS = 16;
constexpr int PER_BLOCK = THREADS * ITEMS;

// Device words: [0] bits of the largest value, [1] unused, [2..3] the first
// index the fixed-point path cannot vouch for (u64, ~0 when none).

__device__ __forceinline__ int ceil_log2_u64(uint64_t x) { return x <= 1 ? 0 : 64 - __clzll(x - 1); }

__device__ __forceinline__ int lsb_exponent(uint32_t maxbits, uint64_t n) {
  int eb = (int)(maxbits >> 23);
  if (eb == 0) eb = 1;
  return eb - 253 + ceil_log2_u64(n + 1);
}

// Exact fixed-point image of a non-negative finite float at weight 2^L.
__device__ __forceinline__ bool to_fixed(float f, int L, u128& out) {
  uint32_t b = __float_as_uint(f);
  if (b == 0u || b == 0x80000000u) {
    out = 0;
    return true;
  }
  if ((b >> 31) || ((b >> 23) & 0xFF) == 0xFF) {
    out = 0;
    return false;
  }
  uint32_t e = b >> 23, m = b & 0x7FFFFFu;
  int ew;
  if (e == 0) {
    ew = -149;
  } else {
    m |= 0x800000u;
    ew = (int)e - 150;
  }
  int sh = ew - L;
  if (sh >= 0) {
    out = (u128)m << sh;
    return true;
  }
  int r = -sh;
  if (r >= 32) {
    out = 0;
    return false;
  }
  out = (u128)(m >> r);
  return (m & ((1u << r) - 1u)) == 0u;
}

__device__ __forceinline__ int clz128(u128 x) {
  uint64_t hi = (uint64_t)(x >> 64), lo = (uint64_t)x;
  return hi ? __clzll(hi) : 64 + __clzll(lo);
}
__device__ __forceinline__ int ctz128(u128 x) {
  uint64_t hi = (uint64_t)(x >> 64), lo = (uint64_t)x;
  return lo ? __ffsll(lo) - 1 : 64 + __ffsll(hi) - 1;
}
__device__ __forceinline__ bool f64_exact(u128 x) {
  if (x == 0) return true;
  return 128 - clz128(x) - ctz128(x) <= 53;
}
// Exact conversion; only called on values that pass f64_exact.
__device__ __forceinline__ double to_double(u128 x, int L) {
  if (x == 0) return 0.0;
  int tz = ctz128(x);
  uint64_t m = (uint64_t)(x >> tz);  // < 2^53
  return ldexp((double)m, tz + L);
}

__device__ __forceinline__ u128 shfl_up_u128(u128 v, int d) {
  uint64_t lo = __shfl_up_sync(0xFFFFFFFFu, (uint64_t)v, d);
  uint64_t hi = __shfl_up_sync(0xFFFFFFFFu, (uint64_t)(v >> 64), d);
  return ((u128)hi << 64) | lo;
}

__device__ __forceinline__ void mark_bad(uint32_t* words, uint64_t i) {
  atomicMin(reinterpret_cast<unsigned long long*>(words + 2), (unsigned long long)i);
}

// Pass 1: largest value (as bits; values are >= 0) and negative / non-finite
// values, which the fixed-point path does not take.
__global__ void max_kernel(const float* __restrict__ v, uint64_t n, uint32_t* words) {
  uint32_t m = 0;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t b = __float_as_uint(v[i]);
    if (b == 0x80000000u) b = 0;
    if ((b >> 31) || ((b >> 23) & 0xFF) == 0xFF)
      mark_bad(words, i);
    else
      m = max(m, b);
  }
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  if ((threadIdx.x & 31) == 0) atomicMax(words, m);
}

// Pass 2: per-block totals of the fixed-point values.
__global__ void __launch_bounds__(THREADS) block_total_kernel(const float* __restrict__ v, uint64_t n,
                                                              uint32_t* words, u128* block_tot) {
  const int L = lsb_exponent(words[0], n);
  const uint64_t base = (uint64_t)blockIdx.x * PER_BLOCK + (uint64_t)threadIdx.x * ITEMS;
  u128 s = 0;
#pragma unroll
  for (int j = 0; j < ITEMS; ++j) {
    uint64_t i = base + j;
    if (i < n) {
      u128 f;
      if (!to_fixed(v[i], L, f)) mark_bad(words, i);
      s += f;
    }
  }
  __shared__ u128 part[THREADS / 32];
  for (int d = 16; d >= 1; d >>= 1) {
    uint64_t lo = __shfl_down_sync(0xFFFFFFFFu, (uint64_t)s, d);
    uint64_t hi = __shfl_down_sync(0xFFFFFFFFu, (uint64_t)(s >> 64), d);
    s += ((u128)hi << 64) | lo;
  }
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    u128 t = 0;
    for (int w = 0; w < THREADS / 32; ++w) t += part[w];
    block_tot[blockIdx.x] = t;
  }
}

// Pass 3: exclusive scan of the block totals (one thread; a few hundred blocks).
__global__ void block_scan_kernel(const u128* block_tot, u128* block_base, uint32_t nblocks) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  u128 run = 0;
  for (uint32_t b = 0; b < nblocks; ++b) {
    block_base[b] = run;
    run += block_tot[b];
  }
}

// Pass 4: every inclusive prefix; records the first one an f64 cannot hold
// and, when asked, stores the prefixes for the cumulative search.
__global__ void __launch_bounds__(THREADS) prefix_kernel(const float* __restrict__ v, uint64_t n, uint32_t* words,
                                                         const u128* __restrict__ block_base, u128* prefix) {
  const int L = lsb_exponent(words[0], n);
  const uint64_t base = (uint64_t)blockIdx.x * PER_BLOCK + (uint64_t)threadIdx.x * ITEMS;
  u128 f[ITEMS];
  u128 s = 0;
#pragma unroll
  for (int j = 0; j < ITEMS; ++j) {
    uint64_t i = base + j;
    f[j] = 0;
    if (i < n) to_fixed(v[i], L, f[j]);
    s += f[j];
  }
  // block-wide exclusive scan of the per-thread sums
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  u128 inc = s;
  for (int d = 1; d < 32; d <<= 1) {
    u128 o = shfl_up_u128(inc, d);
    if (lane >= d) inc += o;
  }
  __shared__ u128 wsum[THREADS / 32];
  if (lane == 31) wsum[warp] = inc;
  __syncthreads();
  u128 wbase = block_base[blockIdx.x];
  for (int w = 0; w < warp; ++w) wbase += wsum[w];
  u128 run = wbase + inc - s;
  uint64_t first_bad = ~0ull;
#pragma unroll
  for (int j = 0; j < ITEMS; ++j) {
    uint64_t i = base + j;
    if (i < n) {
      run += f[j];
      if (prefix) prefix[i] = run;
      if (first_bad == ~0ull && !f64_exact(run)) first_bad = i;
    }
  }
  if (first_bad != ~0ull) mark_bad(words, first_bad);
}

// s_{i0-1}: the exact partial sum just before the first index the fixed-point
// path cannot vouch for.
__device__ inline double exact_prefix_before(const float* v, uint64_t n, uint64_t i0, const uint32_t* words,
                                             const u128* block_base, const u128* prefix) {
  if (i0 == 0) return 0.0;
  const int L = lsb_exponent(words[0], n);
  if (prefix) return to_double(prefix[i0 - 1], L);
  uint64_t b = (i0 - 1) / PER_BLOCK;
  u128 s = block_base[b];
  for (uint64_t i = b * PER_BLOCK; i < i0; ++i) {
    u128 f;
    to_fixed(v[i], L, f);
    s += f;
  }
  return to_double(s, L);
}

// Total: exact when no index is bad, else exact up to i0 and then the
// reference's own loop.
__global__ void total_kernel(const float* __restrict__ v, uint64_t n, const uint32_t* words,
                             const u128* block_base, const u128* block_tot, uint32_t nblocks,
                             const u128* prefix, double* result) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint64_t bad = *reinterpret_cast<const unsigned long long*>(words + 2);
  const uint64_t i0 = bad < n ? bad : n;
  double s;
  if (i0 >= n) {
    const int L = lsb_exponent(words[0], n);
    s = n ? to_double(block_base[nblocks - 1] + block_tot[nblocks - 1], L) : 0.0;
  } else {
    s = exact_prefix_before(v, n, i0, words, block_base, prefix);
    for (uint64_t i = i0; i < n; ++i) s = __dadd_rn(s, (double)v[i]);
  }
  result[0] = s;
}

// Cumulative search: the first i whose running sum reaches `target`, else n-1
// (kmeans.rs:170-177). Needs the stored prefixes.
__global__ void search_kernel(const float* __restrict__ v, uint64_t n, const uint32_t* words,
                              const u128* __restrict__ prefix, double target, unsigned long long* out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint64_t bad = *reinterpret_cast<const unsigned long long*>(words + 2);
  const uint64_t i0 = bad < n ? bad : n;
  const int L = lsb_exponent(words[0], n);
  uint64_t lo = 0, hi = i0;  // first i in [0, i0) with prefix >= target
  while (lo < hi) {
    uint64_t mid = lo + (hi - lo) / 2;
    if (to_double(prefix[mid], L) >= target)
      hi = mid;
    else
      lo = mid + 1;
  }
  if (lo < i0) {
    *out = lo;
    return;
  }
  double s = i0 ? to_double(prefix[i0 - 1], L) : 0.0;
  for (uint64_t i = i0; i < n; ++i) {
    s = __dadd_rn(s, (double)v[i]);
    if (s >= target) {
      *out = i;
      return;
    }
  }
  *out = n ? n - 1 : 0;
}

// Host side: buffers sized for n values.
struct Summer {
  DBuf<uint32_t> words;
  DBuf<u128> tot, base, prefix;
  DBuf<double> result;
  DBuf<unsigned long long> found;
  uint32_t nblocks = 0;

  void reserve(uint64_t n, bool keep_prefix) {
    nblocks = (uint32_t)std::max<uint64_t>(1, (n + PER_BLOCK - 1) / PER_BLOCK);
    words.reserve(4);
    tot.reserve(nblocks);
    base.reserve(nblocks);
    result.reserve(2);
    found.reserve(1);
    if (keep_prefix) prefix.reserve(std::max<uint64_t>(n, 1));
  }
  // Enqueues the sum of v[0..n) into result.p[0]; keep_prefix stores the
  // prefixes for a following search(). Returns the number of kernels launched.
  int enqueue(const float* v, uint64_t n, bool keep_prefix, cudaStream_t s, int sms) {
    reserve(n, keep_prefix);
    PXC_CUDA(cudaMemsetAsync(words.p, 0, 2 * sizeof(uint32_t), s));
    PXC_CUDA(cudaMemsetAsync(words.p + 2, 0xFF, 2 * sizeof(uint32_t), s));
    uint32_t grid = (uint32_t)std::min<uint64_t>((n + 255) / 256 + 1, (uint64_t)sms * 8);
    max_kernel<<<grid, 256, 0, s>>>(v, n, words.p);
    block_total_kernel<<<nblocks, THREADS, 0, s>>>(v, n, words.p, tot.p);
    block_scan_kernel<<<1, 32, 0, s>>>(tot.p, base.p, nblocks);
    prefix_kernel<<<nblocks, THREADS, 0, s>>>(v, n, words.p, base.p, keep_prefix ? prefix.p : nullptr);
    total_kernel<<<1, 32, 0, s>>>(v, n, words.p, base.p, tot.p, nblocks, keep_prefix ? prefix.p : nullptr,
                                  result.p);
    PXC_CUDA(cudaGetLastError());
    return 5;
  }
  int enqueue_search(const float* v, uint64_t n, double target, cudaStream_t s) {
    search_kernel<<<1, 32, 0, s>>>(v, n, words.p, prefix.p, target, found.p);
    PXC_CUDA(cudaGetLastError());
    return 1;
  }
};

}  // namespace seqsum
}  // namespace pxc
