// sq.cu — ScalarQuantizer on the device and the scalar-quantized filtered
// search (int8 over-fetch, exact re-rank).
//
// ScalarQuantizer (crates/proxima-quantize/src/scalar.rs):
//   * train (:141-195): per-group min and max of the training rows. The
//     reference folds `min = min.min(v)` in row-major order; with finite
//     values that keeps the FIRST value of the smallest class, which matters
//     only for the sign of a zero bound. The device takes the class by an
//     atomic minimum over an order key that merges -0 and +0, and the sign
//     of a zero result from the first -0 / +0 seen (atomic minimum of the
//     element index), so the result is bit-identical to the sequential fold;
//   * encode_into (:246-268): level = round_half_away((v - min) * inv)
//     clamped to [0, 255] (NaN to 0, as `as u8` saturates), I8 stores
//     level - 128 (wrapping);
//   * decode (:270-296 reconstruct): min + level * scale.
//
// Filtered search (new composition; the reference has no SQ index, its SQ
// path is train -> encode -> asymmetric scoring, tests/recall.rs:139-148):
//   1. the accepted rows (live, bitmap over slots, integer range filters on
//      metadata columns) are compacted in ascending rank (VectorId) order and
//      their I8 codes gathered contiguously;
//   2. each query is taken to code space, w_c = q_c * scale_g, and quantized
//      to s8 with one step per query (amax / 127);
//   3. K12 (sq_tc.cuh): S = q8 . code on tcgen05 s8 MMA; the top
//      F = max(overfetch, k) columns by (S desc, rank asc). A DENSE pass over
//      a prefix of the columns gives each query its prefix top-F; a THRESH
//      pass over the rest appends only the columns whose key is at or below
//      an admission key, and a block radix select keeps the best F of the
//      union. The admission key is speculative, the r-th prefix key with r
//      sized so that about 4F columns are expected to pass; the result is
//      exact whenever F keys of the union are at or below it, which the
//      merge verifies. Queries that fail are scanned again with the F-th
//      prefix key (always exact), and a query whose candidate buffer still
//      overflows is answered by DENSE passes over all columns;
//   4. exact re-rank of those rows with the reference's distance
//      (cosine 1 - dot_unrolled, inner product -dot_unrolled) and the k
//      smallest by (total_cmp, id).
// The device layout: prepared rows in slot order (the re-rank store), I8
// codes in rank order with a 128-byte-multiple pitch (zero padded), the rank
// -> slot map and per-slot VectorIds, metadata columns as int64 per slot.
#include <cub/device/device_select.cuh>
#include <thrust/iterator/counting_iterator.h>
#include <cuda_pipeline.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <map>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "refdist.cuh"
#include "select.cuh"
#include "sq_tc.cuh"
#include "tmap.cuh"
#include "topk.cuh"

namespace pxc {
namespace sq {

constexpr uint32_t PREFIX = 4096;         // columns of the DENSE prefix pass
constexpr uint64_t SPEC_MARGIN = 4;       // expected admitted columns / F under the speculative key
constexpr uint32_t QBATCH = 4096;         // queries per scan batch
constexpr uint32_t CB = 8192;             // merge buffer (keys) per query
constexpr uint32_t MAX_OVERFETCH = 2048;  // max(overfetch, k)
constexpr uint32_t MAX_DIM = 1024;
constexpr uint32_t MAX_RANGES = 8;

// ---------------------------------------------------------------------------
// train: per-group ranges
// ---------------------------------------------------------------------------
// Order key with -0 and +0 merged (the class the strict comparisons see).
__device__ __forceinline__ uint32_t class_key(float v) { return order_key(v == 0.0f ? 0.0f : v); }

struct RangeOut {
  uint32_t* kmin;           // [groups] class key of the minimum (init ~0)
  uint32_t* kmax;           // [groups] class key of the maximum (init 0)
  unsigned long long* zneg;  // [groups] first element index holding -0 (init ~0)
  unsigned long long* zpos;  // [groups] first element index holding +0 (init ~0)
  unsigned long long* bad;   // first element index that is not finite (init ~0)
};

// Block = 8 warps over the same 32 columns (blockIdx.y), rows of the block's
// range interleaved by warp; each thread folds its column in row order.
__global__ void __launch_bounds__(256) range_kernel(const float* __restrict__ X, uint64_t ld,
                                                   const uint32_t* __restrict__ row_map, uint64_t n,
                                                   uint32_t dim, int global, uint64_t rows_per_block,
                                                   RangeOut o) {
  __shared__ uint32_t s_min[8][32], s_max[8][32];
  __shared__ unsigned long long s_zn[8][32], s_zp[8][32];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t c = blockIdx.y * 32 + lane;
  const uint64_t r0 = blockIdx.x * rows_per_block;
  const uint64_t r1 = min(n, r0 + rows_per_block);
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0;
  unsigned long long zn = ~0ull, zp = ~0ull, bad = ~0ull;
  if (c < dim) {
    for (uint64_t r = r0 + warp; r < r1; r += 8) {
      const float v = __ldg(X + (row_map ? (uint64_t)row_map[r] : r) * ld + c);
      const unsigned long long idx = r * dim + c;
      if (!isfinite(v)) {
        bad = min(bad, idx);
        continue;
      }
      const uint32_t k = class_key(v);
      kmin = min(kmin, k);
      kmax = max(kmax, k);
      if (v == 0.0f) {
        if (signbit(v)) zn = min(zn, idx);
        else zp = min(zp, idx);
      }
    }
  }
  if (bad != ~0ull) atomicMin(o.bad, bad);
  s_min[warp][lane] = kmin;
  s_max[warp][lane] = kmax;
  s_zn[warp][lane] = zn;
  s_zp[warp][lane] = zp;
  __syncthreads();
  if (warp == 0 && c < dim) {
    for (int w = 1; w < 8; ++w) {
      kmin = min(kmin, s_min[w][lane]);
      kmax = max(kmax, s_max[w][lane]);
      zn = min(zn, s_zn[w][lane]);
      zp = min(zp, s_zp[w][lane]);
    }
    const uint32_t g = global ? 0 : c;
    atomicMin(o.kmin + g, kmin);
    atomicMax(o.kmax + g, kmax);
    if (zn != ~0ull) atomicMin(o.zneg + g, zn);
    if (zp != ~0ull) atomicMin(o.zpos + g, zp);
  }
}

// The same for dim % 4 == 0: each lane folds four adjacent columns read as one
// 16-byte load, four rows in flight; a warp covers 128 columns.
__global__ void __launch_bounds__(256) range4_kernel(const float* __restrict__ X, uint64_t ld,
                                                    const uint32_t* __restrict__ row_map, uint64_t n,
                                                    uint32_t dim, int global, uint64_t rows_per_block,
                                                    RangeOut o) {
  __shared__ uint32_t s_min[8][128], s_max[8][128];
  __shared__ unsigned long long s_zn[8][128], s_zp[8][128];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t c0 = blockIdx.y * 128 + lane * 4;
  const uint64_t r0 = blockIdx.x * rows_per_block;
  const uint64_t r1 = min(n, r0 + rows_per_block);
  uint32_t kmin[4], kmax[4];
  unsigned long long zn[4], zp[4], bad = ~0ull;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    kmin[u] = 0xFFFFFFFFu;
    kmax[u] = 0;
    zn[u] = zp[u] = ~0ull;
  }
  auto fold = [&](float v, uint64_t r, int u) {
    const unsigned long long idx = r * dim + c0 + u;
    if (!isfinite(v)) {
      bad = min(bad, idx);
      return;
    }
    const uint32_t k = class_key(v);
    kmin[u] = min(kmin[u], k);
    kmax[u] = max(kmax[u], k);
    if (v == 0.0f) {
      if (signbit(v)) zn[u] = min(zn[u], idx);
      else zp[u] = min(zp[u], idx);
    }
  };
  if (c0 < dim) {
    uint64_t r = r0 + warp;
    for (; r + 24 < r1; r += 32) {  // four rows of this warp in flight, folded in row order
      float4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint64_t rr = r + 8 * j;
        v[j] = __ldg(reinterpret_cast<const float4*>(X + (row_map ? (uint64_t)row_map[rr] : rr) * ld + c0));
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        fold(v[j].x, r + 8 * j, 0);
        fold(v[j].y, r + 8 * j, 1);
        fold(v[j].z, r + 8 * j, 2);
        fold(v[j].w, r + 8 * j, 3);
      }
    }
    for (; r < r1; r += 8) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(X + (row_map ? (uint64_t)row_map[r] : r) * ld + c0));
      fold(v.x, r, 0);
      fold(v.y, r, 1);
      fold(v.z, r, 2);
      fold(v.w, r, 3);
    }
  }
  if (bad != ~0ull) atomicMin(o.bad, bad);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    s_min[warp][lane * 4 + u] = kmin[u];
    s_max[warp][lane * 4 + u] = kmax[u];
    s_zn[warp][lane * 4 + u] = zn[u];
    s_zp[warp][lane * 4 + u] = zp[u];
  }
  __syncthreads();
  if (threadIdx.x < 128) {
    const uint32_t cc = threadIdx.x, c = blockIdx.y * 128 + cc;
    if (c < dim) {
      uint32_t mn = s_min[0][cc], mx = s_max[0][cc];
      unsigned long long a = s_zn[0][cc], b = s_zp[0][cc];
      for (int w = 1; w < 8; ++w) {
        mn = min(mn, s_min[w][cc]);
        mx = max(mx, s_max[w][cc]);
        a = min(a, s_zn[w][cc]);
        b = min(b, s_zp[w][cc]);
      }
      const uint32_t g = global ? 0 : c;
      atomicMin(o.kmin + g, mn);
      atomicMax(o.kmax + g, mx);
      if (a != ~0ull) atomicMin(o.zneg + g, a);
      if (b != ~0ull) atomicMin(o.zpos + g, b);
    }
  }
}

// ---------------------------------------------------------------------------
// encode / decode
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint8_t encode_one(float v, float mn, float inv, int i8) {
  float x = roundf(__fmul_rn(__fsub_rn(v, mn), inv));
  x = !(x >= 0.0f) ? 0.0f : (x > 255.0f ? 255.0f : x);
  const uint8_t level = static_cast<uint8_t>(x);
  return i8 ? static_cast<uint8_t>(level ^ 0x80u) : level;
}

// codes[r][0..pitch) from row src(r) (row_map ? row_map[r] : r); columns past
// dim are zero.
__global__ void __launch_bounds__(256) encode_kernel(const float* __restrict__ X, uint64_t ld,
                                                     const uint32_t* __restrict__ row_map, uint64_t n,
                                                     uint32_t dim, const float* __restrict__ mn,
                                                     const float* __restrict__ inv, int global, int i8,
                                                     uint8_t* __restrict__ codes, uint64_t pitch) {
  for (uint64_t r = blockIdx.y; r < n; r += gridDim.y) {
    const uint64_t src = row_map ? row_map[r] : r;
    const float* x = X + src * ld;
    uint8_t* out = codes + r * pitch;
    for (uint64_t c = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; c < pitch;
         c += (uint64_t)gridDim.x * blockDim.x) {
      uint8_t b = 0;
      if (c < dim) {
        const uint32_t g = global ? 0 : (uint32_t)c;
        b = encode_one(__ldg(x + c), mn[g], inv[g], i8);
      }
      out[c] = b;
    }
  }
}

// Same for dim % 4 == 0, ld % 4 == 0, pitch % 4 == 0: four columns per thread.
__global__ void __launch_bounds__(256) encode4_kernel(const float* __restrict__ X, uint64_t ld,
                                                      const uint32_t* __restrict__ row_map, uint64_t n,
                                                      uint32_t dim, const float* __restrict__ mn,
                                                      const float* __restrict__ inv, int global, int i8,
                                                      uint8_t* __restrict__ codes, uint64_t pitch) {
  const uint32_t quads = (uint32_t)(pitch / 4);
  for (uint64_t r = blockIdx.y; r < n; r += gridDim.y) {
    const uint64_t src = row_map ? row_map[r] : r;
    const float4* x = reinterpret_cast<const float4*>(X + src * ld);
    uchar4* out = reinterpret_cast<uchar4*>(codes + r * pitch);
    for (uint32_t c4 = blockIdx.x * blockDim.x + threadIdx.x; c4 < quads; c4 += gridDim.x * blockDim.x) {
      uchar4 b = make_uchar4(0, 0, 0, 0);
      const uint32_t c = 4 * c4;
      if (c < dim) {
        const float4 v = __ldg(x + c4);
        const uint32_t g0 = global ? 0 : c;
        const uint32_t g1 = global ? 0 : c + 1, g2 = global ? 0 : c + 2, g3 = global ? 0 : c + 3;
        b.x = encode_one(v.x, mn[g0], inv[g0], i8);
        b.y = encode_one(v.y, mn[g1], inv[g1], i8);
        b.z = encode_one(v.z, mn[g2], inv[g2], i8);
        b.w = encode_one(v.w, mn[g3], inv[g3], i8);
      }
      out[c4] = b;
    }
  }
}

__global__ void __launch_bounds__(256) decode_kernel(const uint8_t* __restrict__ codes, uint64_t n, uint32_t dim,
                                                     const float* __restrict__ mn, const float* __restrict__ sc,
                                                     int global, int i8, float* __restrict__ out) {
  const uint64_t total = n * dim;
  for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t c = (uint32_t)(e % dim);
    const uint32_t g = global ? 0 : c;
    const uint8_t level = i8 ? static_cast<uint8_t>(codes[e] ^ 0x80u) : codes[e];
    out[e] = __fadd_rn(mn[g], __fmul_rn(static_cast<float>(level), sc[g]));
  }
}

// ScalarQuantizer::asymmetric_squared_l2 / asymmetric_inner_product
// (scalar.rs:298-327) for every (query, code) pair: the sequential sum over
// components of d * d with d = q - reconstruct, or of q * reconstruct then
// negated, where reconstruct = min + f32(level) * scale; every step rounded
// on its own (no contraction), as the reference computes it. Block = 128
// codes (one per thread) x ASYM_Q queries; each 64-component slab of the
// codes and queries is staged in shared memory, so one reconstruct serves
// ASYM_Q queries. out[q * n + row].
constexpr uint32_t ASYM_Q = 8;
constexpr uint32_t ASYM_SLAB = 64;
__global__ void __launch_bounds__(128) asymmetric_kernel(const float* __restrict__ Q, uint32_t nq,
                                                         const uint8_t* __restrict__ codes, uint64_t n,
                                                         uint32_t dim, const float* __restrict__ mn,
                                                         const float* __restrict__ sc, int global, int i8,
                                                         int inner, float* __restrict__ out) {
  __shared__ uint8_t s_codes[128][ASYM_SLAB + 4];  // 68-byte rows: a warp's reads of one column hit distinct banks
  __shared__ float s_q[ASYM_Q][ASYM_SLAB];
  const uint64_t row0 = (uint64_t)blockIdx.x * 128;
  const uint32_t q0 = blockIdx.y * ASYM_Q;
  const uint32_t nqb = min(ASYM_Q, nq - q0);
  float sum[ASYM_Q];
#pragma unroll
  for (int j = 0; j < (int)ASYM_Q; ++j) sum[j] = 0.0f;
  for (uint32_t c0 = 0; c0 < dim; c0 += ASYM_SLAB) {
    const uint32_t w = min(ASYM_SLAB, dim - c0);
    __syncthreads();
    for (uint32_t e = threadIdx.x; e < 128 * w; e += 128) {
      const uint32_t r = e / w, t = e - r * w;
      const uint64_t gr = row0 + r;
      s_codes[r][t] = gr < n ? codes[gr * dim + c0 + t] : 0;
    }
    for (uint32_t e = threadIdx.x; e < ASYM_Q * w; e += 128) {
      const uint32_t j = e / w, t = e - j * w;
      s_q[j][t] = j < nqb ? Q[(size_t)(q0 + j) * dim + c0 + t] : 0.0f;
    }
    __syncthreads();
    for (uint32_t t = 0; t < w; ++t) {
      const uint32_t c = c0 + t, g = global ? 0 : c;
      const uint8_t b = s_codes[threadIdx.x][t];
      const uint8_t level = i8 ? static_cast<uint8_t>(b ^ 0x80u) : b;
      const float r = __fadd_rn(__ldg(mn + g), __fmul_rn(static_cast<float>(level), __ldg(sc + g)));
#pragma unroll
      for (int j = 0; j < (int)ASYM_Q; ++j) {
        const float qv = s_q[j][t];
        if (inner) {
          sum[j] = __fadd_rn(sum[j], __fmul_rn(qv, r));
        } else {
          const float d = __fsub_rn(qv, r);
          sum[j] = __fadd_rn(sum[j], __fmul_rn(d, d));
        }
      }
    }
  }
  const uint64_t row = row0 + threadIdx.x;
  if (row >= n) return;
  for (uint32_t j = 0; j < nqb; ++j) out[(size_t)(q0 + j) * n + row] = inner ? -sum[j] : sum[j];
}

// ---------------------------------------------------------------------------
// search: acceptance, compaction, query preparation
// ---------------------------------------------------------------------------
struct RangeFilter {
  const int64_t* values[MAX_RANGES];
  const uint8_t* present[MAX_RANGES];  // nullable: every slot has the field
  int64_t lo[MAX_RANGES], hi[MAX_RANGES];
  uint32_t n;
};

__global__ void accept_kernel(const uint32_t* __restrict__ rank_slot, uint64_t nrank,
                              const uint64_t* __restrict__ bitmap, RangeFilter f, uint8_t* __restrict__ flags) {
  for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < nrank; r += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t slot = rank_slot[r];
    bool ok = bitmap == nullptr || ((bitmap[slot >> 6] >> (slot & 63)) & 1ull);
    for (uint32_t j = 0; j < f.n && ok; ++j) {
      if (f.present[j] && !f.present[j][slot]) ok = false;
      else {
        const int64_t v = f.values[j][slot];
        ok = v >= f.lo[j] && v <= f.hi[j];
      }
    }
    flags[r] = ok ? 1 : 0;
  }
}

// dst row i = src row idx[i] (pitch bytes, a multiple of 16).
__global__ void gather_rows16_kernel(const uint8_t* __restrict__ src, const uint32_t* __restrict__ idx,
                                     const uint32_t* __restrict__ d_count, uint64_t count_cap, uint64_t pitch,
                                     uint8_t* __restrict__ dst) {
  const uint64_t count = d_count ? min((uint64_t)*d_count, count_cap) : count_cap;
  const uint64_t per = pitch / 16;
  const uint64_t total = count * per;
  for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = e / per, w = e % per;
    reinterpret_cast<uint4*>(dst + i * pitch)[w] = __ldg(reinterpret_cast<const uint4*>(src + (uint64_t)idx[i] * pitch) + w);
  }
}

// Queries to code space: w_c = q_c * scale_g; q8_c = clamp(round(w_c * (127 /
// amax)), -127, 127). Rows past nq and columns past dim are zero. One block
// per (padded) query.
__global__ void __launch_bounds__(256) query_s8_kernel(const float* __restrict__ Q, uint32_t nq, uint32_t dim,
                                                       const float* __restrict__ scale, int global,
                                                       int8_t* __restrict__ q8, uint32_t pitch) {
  __shared__ float red[8];
  const uint32_t q = blockIdx.x;
  int8_t* out = q8 + (size_t)q * pitch;
  if (q >= nq) {
    for (uint32_t c = threadIdx.x; c < pitch; c += blockDim.x) out[c] = 0;
    return;
  }
  const float* qv = Q + (size_t)q * dim;
  float amax = 0.0f;
  for (uint32_t c = threadIdx.x; c < dim; c += blockDim.x)
    amax = fmaxf(amax, fabsf(__fmul_rn(qv[c], scale[global ? 0 : c])));
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = red[0];
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
  const float inv = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
  for (uint32_t c = threadIdx.x; c < pitch; c += blockDim.x) {
    int8_t b = 0;
    if (c < dim) {
      float x = roundf(__fmul_rn(__fmul_rn(qv[c], scale[global ? 0 : c]), inv));
      x = x < -127.0f ? -127.0f : (x > 127.0f ? 127.0f : x);
      b = static_cast<int8_t>(x);
    }
    out[c] = b;
  }
}

// Top F of the prefix pass per query (block of PSEL_THREADS threads), in
// place of a general chunk selection: the keys of columns [0, p0) are read
// from the DENSE matrix into registers; one histogram over their observed
// range (256 bins, warp-private counters) finds the bin holding the F-th key;
// only keys in that bin or below survive into shared memory as
// (key << 32 | column), an exact radix select keeps F of them, and they are
// sorted. Writes L0 (ascending), len0, and the admission keys tau_spec (the
// r-th) and tau_safe (the F-th); both are SENTINEL when fewer than F columns
// exist.
constexpr uint32_t PSEL_THREADS = 256;
constexpr uint32_t PSEL_PER = PREFIX / PSEL_THREADS;
__global__ void __launch_bounds__(PSEL_THREADS) prefix_select_kernel(const uint32_t* __restrict__ D, uint64_t ld,
                                                                     uint32_t p0, uint32_t F, uint32_t r,
                                                                     uint64_t* __restrict__ L0, uint32_t* __restrict__ len0,
                                                                     uint32_t* __restrict__ tau_spec,
                                                                     uint32_t* __restrict__ tau_safe) {
  extern __shared__ __align__(16) uint64_t buf[];  // CB entries
  __shared__ uint32_t hist[PSEL_THREADS / 32][256];
  __shared__ uint32_t tot[256], hsel[256], sh[4];
  __shared__ uint32_t s_min, s_max, s_bin, s_cnt;
  const uint32_t q = blockIdx.x, t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const uint32_t* Dq = D + (size_t)q * ld;
  uint32_t k[PSEL_PER];
  uint32_t mn = 0xFFFFFFFFu, mx = 0;
#pragma unroll
  for (uint32_t i = 0; i < PSEL_PER; ++i) {
    const uint32_t c = t + i * PSEL_THREADS;
    k[i] = c < p0 ? Dq[c] : SENTINEL;
    if (k[i] != SENTINEL) {
      mn = min(mn, k[i]);
      mx = max(mx, k[i]);
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    mn = min(mn, __shfl_xor_sync(0xFFFFFFFFu, mn, o));
    mx = max(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
  }
  if (t == 0) {
    s_min = 0xFFFFFFFFu;
    s_max = 0;
    s_cnt = 0;
  }
  for (uint32_t b = t; b < 256 * (PSEL_THREADS / 32); b += PSEL_THREADS) (&hist[0][0])[b] = 0;
  __syncthreads();
  if (lane == 0) {
    atomicMin(&s_min, mn);
    atomicMax(&s_max, mx);
  }
  __syncthreads();
  const uint32_t kmin = s_min, span = s_max - s_min;
  const uint32_t shift = (s_max < s_min || span < 256) ? 0u : (32u - __clz(span)) - 8u;
#pragma unroll
  for (uint32_t i = 0; i < PSEL_PER; ++i)
    if (k[i] != SENTINEL) atomicAdd(&hist[warp][(k[i] - kmin) >> shift], 1u);
  __syncthreads();
  {
    uint32_t sum = 0;
    for (uint32_t w = 0; w < PSEL_THREADS / 32; ++w) sum += hist[w][t & 255];
    if (t < 256) tot[t] = sum;
  }
  __syncthreads();
  if (warp == 0) {  // prefix sums over the 256 bins: the bin holding the F-th key
    uint32_t c[8], ssum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = tot[lane * 8 + j];
      ssum += c[j];
    }
    uint32_t inc = ssum;
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
      if (lane >= (uint32_t)o) inc += v;
    }
    const uint32_t total = __shfl_sync(0xFFFFFFFFu, inc, 31);
    if (lane == 0 && total < F) s_bin = 255;  // fewer than F keys: every one survives
    uint32_t before = inc - ssum;
    if (total >= F && before < F && inc >= F) {
      uint32_t acc = before;
      for (int j = 0; j < 8; ++j) {
        acc += c[j];
        if (acc >= F) {
          s_bin = lane * 8 + j;
          break;
        }
      }
    }
  }
  __syncthreads();
  const uint32_t bstar = s_bin;
#pragma unroll
  for (uint32_t i = 0; i < PSEL_PER; ++i) {
    if (k[i] != SENTINEL && ((k[i] - kmin) >> shift) <= bstar)
      buf[atomicAdd(&s_cnt, 1u)] = (static_cast<uint64_t>(k[i]) << 32) | (t + i * PSEL_THREADS);
  }
  __syncthreads();
  const uint32_t n = s_cnt;
  uint32_t keep = n;
  if (n > F) {
    select_keep<CB / PSEL_THREADS>(buf, n, F, hsel, sh);
    keep = F;
  }
  uint32_t n2 = 1;
  while (n2 < keep) n2 <<= 1;
  for (uint32_t i = keep + t; i < n2; i += PSEL_THREADS) buf[i] = ~0ull;
  block_bitonic_sort_u64(buf, n2);
  for (uint32_t i = t; i < keep; i += PSEL_THREADS) L0[(size_t)q * F + i] = buf[i];
  if (t == 0) {
    len0[q] = keep;
    const bool full = keep >= F;
    tau_spec[q] = full ? static_cast<uint32_t>(buf[r - 1] >> 32) : SENTINEL;
    tau_safe[q] = full ? static_cast<uint32_t>(buf[F - 1] >> 32) : SENTINEL;
  }
}

__global__ void gather_u32_kernel(const uint32_t* __restrict__ src, const uint32_t* __restrict__ idx, uint32_t n,
                                  uint32_t* __restrict__ dst) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[idx[i]];
}

// Per query: the union of its prefix list and its THRESH candidates, cut to
// the best F (candidates taken CB - F at a time, the kept F carried over).
// The query is listed in `fail` instead when its candidates overflowed the
// buffer, or (with `verify`) when fewer than F of the union are at or below
// the admission key it was scanned with: only then is the union's top F
// certainly the exact top F. A failed query's `next_tau` is a key with at
// least F columns at or below it (the F-th of the union, or `safe_tau` after
// an overflow), a valid admission key for its next scan.
__global__ void __launch_bounds__(256) merge_kernel(const uint64_t* __restrict__ L0, const uint32_t* __restrict__ len0,
                                                    const uint64_t* __restrict__ cand, const uint32_t* __restrict__ cnt,
                                                    uint32_t cap, uint32_t F, const uint32_t* __restrict__ verify,
                                                    const uint32_t* __restrict__ safe_tau, uint64_t* __restrict__ Lf,
                                                    uint32_t* __restrict__ lenf, uint32_t* __restrict__ next_tau,
                                                    uint32_t* __restrict__ fail, uint32_t* __restrict__ n_fail) {
  extern __shared__ __align__(16) uint64_t buf[];
  __shared__ uint32_t hist[256], sh[4];
  __shared__ unsigned long long s_max;
  const uint32_t q = blockIdx.x;
  const uint32_t c = cnt[q];
  const uint32_t l0 = len0[q];
  if (c > cap || (verify && l0 + c < F)) {
    if (threadIdx.x == 0) {
      lenf[q] = 0;
      if (next_tau) next_tau[q] = safe_tau ? safe_tau[q] : SENTINEL;
      fail[atomicAdd(n_fail, 1u)] = q;
    }
    return;
  }
  for (uint32_t i = threadIdx.x; i < l0; i += blockDim.x) buf[i] = L0[(size_t)q * F + i];
  uint32_t n = l0;
  bool selected = false;
  uint64_t kth = 0;
  for (uint32_t off = 0; off < c; off += CB - F) {
    const uint32_t m = min(CB - F, c - off);
    for (uint32_t i = threadIdx.x; i < m; i += blockDim.x) buf[n + i] = cand[(size_t)q * cap + off + i];
    n += m;
    __syncthreads();
    if (n > F) {
      kth = select_keep<CB / 256>(buf, n, F, hist, sh);
      n = F;
      selected = true;
    }
  }
  if (!selected) {
    if (threadIdx.x == 0) s_max = 0;
    __syncthreads();
    unsigned long long mx = 0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) mx = max(mx, (unsigned long long)buf[i]);
    atomicMax(&s_max, mx);
    __syncthreads();
    kth = s_max;
  }
  if (verify && static_cast<uint32_t>(kth >> 32) > verify[q]) {
    if (threadIdx.x == 0) {
      lenf[q] = 0;
      if (next_tau) next_tau[q] = static_cast<uint32_t>(kth >> 32);
      fail[atomicAdd(n_fail, 1u)] = q;
    }
    return;
  }
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) Lf[(size_t)q * F + i] = buf[i];
  if (threadIdx.x == 0) lenf[q] = n;
}

__global__ void gather_lists_kernel(const uint64_t* __restrict__ L, const uint32_t* __restrict__ len,
                                    const uint32_t* __restrict__ ovf, uint32_t F, uint64_t* __restrict__ Ls,
                                    uint32_t* __restrict__ lens) {
  const uint32_t i = blockIdx.x, q = ovf[i];
  for (uint32_t j = threadIdx.x; j < F; j += blockDim.x) Ls[(size_t)i * F + j] = L[(size_t)q * F + j];
  if (threadIdx.x == 0) lens[i] = len[q];
}

__global__ void scatter_lists_kernel(const uint64_t* __restrict__ Ls, const uint32_t* __restrict__ lens,
                                     const uint32_t* __restrict__ ovf, uint32_t F, uint64_t* __restrict__ L,
                                     uint32_t* __restrict__ len) {
  const uint32_t i = blockIdx.x, q = ovf[i];
  const uint32_t n = lens[i];
  for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) L[(size_t)q * F + j] = Ls[(size_t)i * F + j];
  if (threadIdx.x == 0) len[q] = n;
}

// K2 for SQ: exact distances of a query's <= F candidates and the k
// smallest by (key, rank). Groups of eight threads take one candidate at a
// time: the row is first copied into the group's shared-memory slot with
// asynchronous 16-byte copies (all in flight at once), then thread l runs
// lane l of dot_unrolled over it, the lanes are combined by the same
// pairwise tree and the tail is added.
constexpr uint32_t RR_THREADS = 128;
constexpr uint32_t RR_GROUPS = RR_THREADS / 8;
__host__ __device__ inline uint32_t rr_stride(uint32_t dim) { return (dim + 3) / 4 * 4 + 8; }
__host__ inline size_t rr_smem(uint32_t dim) {
  return (size_t)MAX_OVERFETCH * 8 + (size_t)rr_stride(dim) * 4 * (RR_GROUPS + 1);
}
__global__ void __launch_bounds__(RR_THREADS) rerank_kernel(const float* __restrict__ Q, uint32_t dim,
                                                            const uint64_t* __restrict__ Lf, const uint32_t* __restrict__ lenf,
                                                            uint32_t F, const uint32_t* __restrict__ acc,
                                                            const uint32_t* __restrict__ rank_slot, const float* __restrict__ rows,
                                                            const uint64_t* __restrict__ ids, int metric, uint32_t k,
                                                            uint64_t* __restrict__ out_ids, float* __restrict__ out_dist,
                                                            uint32_t* __restrict__ out_len) {
  extern __shared__ __align__(16) unsigned char smem[];
  uint64_t* keys = reinterpret_cast<uint64_t*>(smem);  // [MAX_OVERFETCH]
  const uint32_t stride = rr_stride(dim);
  float* qs = reinterpret_cast<float*>(keys + MAX_OVERFETCH);
  float* slots = qs + stride;
  const uint32_t q = blockIdx.x;
  const uint32_t n = lenf[q];
  uint32_t n2 = 1;
  while (n2 < n) n2 <<= 1;
  for (uint32_t c = threadIdx.x; c < dim; c += blockDim.x) qs[c] = Q[(size_t)q * dim + c];
  for (uint32_t i = n + threadIdx.x; i < n2; i += blockDim.x) keys[i] = ~0ull;
  __syncthreads();
  const uint32_t l = threadIdx.x & 7, grp = threadIdx.x >> 3;
  float* slot = slots + (size_t)grp * stride;
  const uint32_t full = dim & ~7u;
  const bool vec = (dim & 3) == 0;
  for (uint32_t base = 0; base < n; base += RR_GROUPS) {
    const uint32_t i = base + grp;
    const bool on = i < n;
    uint32_t rank = 0;
    if (on) {
      const uint32_t col = static_cast<uint32_t>(Lf[(size_t)q * F + i]);
      rank = acc ? acc[col] : col;
      const float* x = rows + (size_t)rank_slot[rank] * dim;
      if (vec) {
        for (uint32_t e = 4 * l; e < dim; e += 32) __pipeline_memcpy_async(slot + e, x + e, 16);
        __pipeline_commit();
        __pipeline_wait_prior(0);
      } else {
        for (uint32_t e = l; e < dim; e += 8) slot[e] = __ldg(x + e);
      }
    }
    __syncwarp();
    float a = 0.0f, tail = 0.0f;
    if (on) {
      for (uint32_t e = l; e < full; e += 8) a = __fadd_rn(a, __fmul_rn(qs[e], slot[e]));
      if (l == 0)
        for (uint32_t e = full; e < dim; ++e) tail = __fadd_rn(tail, __fmul_rn(qs[e], slot[e]));
    }
    // ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)): IEEE addition is commutative, so
    // the xor-butterfly within the group of eight forms exactly these sums.
    a = __fadd_rn(a, __shfl_xor_sync(0xFFFFFFFFu, a, 1));
    a = __fadd_rn(a, __shfl_xor_sync(0xFFFFFFFFu, a, 2));
    a = __fadd_rn(a, __shfl_xor_sync(0xFFFFFFFFu, a, 4));
    if (on && l == 0) {
      const float dot = __fadd_rn(a, tail);
      const float d = metric == PXC_COSINE ? __fsub_rn(1.0f, dot) : -dot;
      keys[i] = (static_cast<uint64_t>(order_key(d)) << 32) | rank;
    }
    __syncwarp();  // the slot is read before the next copy overwrites it
  }
  block_bitonic_sort_u64(keys, n2);
  const uint32_t take = min(n, k);
  for (uint32_t i = threadIdx.x; i < take; i += blockDim.x) {
    const uint64_t key = keys[i];
    out_ids[(size_t)q * k + i] = ids[rank_slot[static_cast<uint32_t>(key)]];
    out_dist[(size_t)q * k + i] = key_to_float(static_cast<uint32_t>(key >> 32));
  }
  if (threadIdx.x == 0) out_len[q] = take;
}

}  // namespace sq
}  // namespace pxc

using namespace pxc;

// ---------------------------------------------------------------------------
// The SQ index handle.
// ---------------------------------------------------------------------------
struct pxc_sq {
  pxc_ctx* ctx = nullptr;
  uint32_t dim = 0, pitch = 0;
  int32_t metric = PXC_COSINE;
  int32_t mode = PXC_RANGE_PER_DIMENSION;
  bool have_quantizer = false;
  std::vector<float> h_min, h_scale, h_inv;
  DBuf<float> d_min, d_scale, d_inv;
  // store
  uint64_t nslots = 0, nrank = 0;
  bool have_rows = false, codes_ready = false;
  DBuf<float> rows;          // nslots x dim, prepared (slot order)
  DBuf<uint64_t> ids;        // nslots
  DBuf<uint32_t> rank_slot;  // nrank
  DBuf<uint8_t> codes;       // nrank x pitch, I8 (rank order)
  std::map<uint32_t, std::pair<DBuf<int64_t>*, DBuf<uint8_t>*>> columns;
  // search scratch (grown on demand)
  DBuf<uint8_t> flags, codes_c, q8, q8s, sel_tmp;
  DBuf<uint32_t> acc, d_nacc, D, len0, lenf, lens, lens2, tau, cnt, ovf, n_ovf;
  DBuf<uint64_t> L0, Lf, Ls, Ls2, L1, L2, cand;
  DBuf<uint32_t> len1, len2;
  DBuf<float> q_dev;
  DBuf<uint64_t> o_ids;
  DBuf<float> o_dist;
  DBuf<uint32_t> o_len;
  uint32_t* h_word = nullptr;  // pinned
  // observability
  cudaEvent_t ev_begin = nullptr, ev_end = nullptr;
  bool timed = false;
  uint64_t last_accepted = 0;
  uint32_t last_fallback = 0;
  uint32_t last_retried = 0;
  std::mutex mu;
  ~pxc_sq() {
    for (auto& c : columns) {
      delete c.second.first;
      delete c.second.second;
    }
    if (h_word) cudaFreeHost(h_word);
    if (ev_begin) cudaEventDestroy(ev_begin);
    if (ev_end) cudaEventDestroy(ev_end);
  }
};

namespace pxc {
namespace sq {

inline uint64_t round_up(uint64_t x, uint64_t m) { return (x + m - 1) / m * m; }

// Per-group (min, max) of n rows (device), bit-identical to the sequential
// fold of ScalarQuantizer::train. Throws PXC_NON_FINITE at the first
// non-finite component (a = its index within the vector, as the reference's
// NonFinite{index} reports).
void ranges_device(pxc_ctx* ctx, const float* d_x, const uint32_t* d_row_map, uint64_t n, uint32_t dim,
                   int32_t mode, float* h_min, float* h_max, cudaStream_t s) {
  PXC_CONFIG(n > 0, "training", 0, "must be a non-empty multiple of the space dimension");
  PXC_CONFIG(dim > 0, "dim", dim, "must be positive");
  PXC_CONFIG(mode == PXC_RANGE_GLOBAL || mode == PXC_RANGE_PER_DIMENSION, "mode", mode, "unknown range mode");
  const uint32_t groups = mode == PXC_RANGE_GLOBAL ? 1 : dim;
  DBuf<uint8_t> ws;
  const size_t bytes = (size_t)groups * 8 + (size_t)groups * 16 + 8;
  ws.reserve(bytes);
  RangeOut o;
  o.kmin = reinterpret_cast<uint32_t*>(ws.p);
  o.kmax = o.kmin + groups;
  o.zneg = reinterpret_cast<unsigned long long*>(ws.p + (size_t)groups * 8);
  o.zpos = o.zneg + groups;
  o.bad = o.zpos + groups;
  PXC_CUDA(cudaMemsetAsync(o.kmin, 0xFF, groups * 4, s));
  PXC_CUDA(cudaMemsetAsync(o.kmax, 0, groups * 4, s));
  PXC_CUDA(cudaMemsetAsync(o.zneg, 0xFF, (size_t)groups * 16 + 8, s));
  const bool vec = dim % 4 == 0 && (reinterpret_cast<uintptr_t>(d_x) & 15) == 0;
  const uint32_t cgroups = vec ? (dim + 127) / 128 : (dim + 31) / 32;
  const uint64_t target_blocks = (uint64_t)ctx->sm_count * 8;
  uint64_t rblocks = std::max<uint64_t>(1, target_blocks / cgroups);
  const uint64_t rows_per_block = std::max<uint64_t>(64, (n + rblocks - 1) / rblocks);
  rblocks = (n + rows_per_block - 1) / rows_per_block;
  if (vec)
    range4_kernel<<<dim3((unsigned)rblocks, cgroups), 256, 0, s>>>(d_x, dim, d_row_map, n, dim,
                                                                    mode == PXC_RANGE_GLOBAL, rows_per_block, o);
  else
    range_kernel<<<dim3((unsigned)rblocks, cgroups), 256, 0, s>>>(d_x, dim, d_row_map, n, dim,
                                                                   mode == PXC_RANGE_GLOBAL, rows_per_block, o);
  PXC_CUDA(cudaGetLastError());
  ctx->launches += 1;
  std::vector<uint8_t> h(bytes);
  PXC_CUDA(cudaMemcpyAsync(h.data(), ws.p, bytes, cudaMemcpyDeviceToHost, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  const uint32_t* kmin = reinterpret_cast<const uint32_t*>(h.data());
  const uint32_t* kmax = kmin + groups;
  const uint64_t* zneg = reinterpret_cast<const uint64_t*>(h.data() + (size_t)groups * 8);
  const uint64_t* zpos = zneg + groups;
  const uint64_t bad = zpos[groups];
  if (bad != ~0ull)
    throw make_failure(PXC_NON_FINITE, bad % dim, 0, "training", "training component %llu is not finite",
                       (unsigned long long)(bad % dim));
  for (uint32_t g = 0; g < groups; ++g) {
    float lo = key_to_float(kmin[g]), hi = key_to_float(kmax[g]);
    // a zero class keeps the sign of its first occurrence
    if (lo == 0.0f) lo = zneg[g] < zpos[g] ? -0.0f : 0.0f;
    if (hi == 0.0f) hi = zneg[g] < zpos[g] ? -0.0f : 0.0f;
    h_min[g] = lo;
    h_max[g] = hi;
  }
}

// scale = (hi - lo) / 255; inverse = scale > 0 ? 1 / scale : 0 (scalar.rs:176-184).
void finish_train(uint32_t groups, const float* lo, const float* hi, float* out_min, float* out_scale, float* out_inv) {
  for (uint32_t g = 0; g < groups; ++g) {
    const float sc = (hi[g] - lo[g]) / 255.0f;
    out_min[g] = lo[g];
    out_scale[g] = sc;
    out_inv[g] = sc > 0.0f ? 1.0f / sc : 0.0f;
  }
}

void encode_device(pxc_ctx* ctx, const float* d_x, uint64_t ld, const uint32_t* d_row_map, uint64_t n, uint32_t dim,
                   const float* d_min, const float* d_inv, int32_t mode, int32_t code_type, uint8_t* d_codes,
                   uint64_t pitch, cudaStream_t s) {
  if (n == 0) return;
  const unsigned gy = (unsigned)std::min<uint64_t>(n, 65535);
  if (dim % 4 == 0 && ld % 4 == 0 && pitch % 4 == 0) {
    const unsigned gx = (unsigned)std::max<uint64_t>(1, (pitch / 4 + 255) / 256);
    encode4_kernel<<<dim3(gx, gy), 256, 0, s>>>(d_x, ld, d_row_map, n, dim, d_min, d_inv, mode == PXC_RANGE_GLOBAL,
                                                 code_type == PXC_CODE_I8, d_codes, pitch);
  } else {
    const unsigned gx = (unsigned)std::max<uint64_t>(1, (pitch + 255) / 256);
    encode_kernel<<<dim3(gx, gy), 256, 0, s>>>(d_x, ld, d_row_map, n, dim, d_min, d_inv, mode == PXC_RANGE_GLOBAL,
                                                code_type == PXC_CODE_I8, d_codes, pitch);
  }
  PXC_CUDA(cudaGetLastError());
  ctx->launches += 1;
}

void check_quantizer_args(uint32_t dim, int32_t mode, int32_t code_type) {
  PXC_CONFIG(dim > 0, "dim", dim, "must be positive");
  PXC_CONFIG(mode == PXC_RANGE_GLOBAL || mode == PXC_RANGE_PER_DIMENSION, "mode", mode, "unknown range mode");
  PXC_CONFIG(code_type == PXC_CODE_U8 || code_type == PXC_CODE_I8, "code_type", code_type, "unknown code type");
}

// Codes of the stored rows, in rank order (both the store and the quantizer
// are needed).
void rebuild_codes(pxc_sq* h, cudaStream_t s) {
  h->codes_ready = false;
  if (!h->have_quantizer || !h->have_rows) return;
  // rows padded to a whole code tile (zero), so every TMA box starts inside the tensor
  const uint64_t rows_pad = round_up(std::max<uint64_t>(1, h->nrank), sq_tc::BN);
  h->codes.reserve(rows_pad * h->pitch);
  PXC_CUDA(cudaMemsetAsync(h->codes.p + h->nrank * h->pitch, 0, (rows_pad - h->nrank) * h->pitch, s));
  encode_device(h->ctx, h->rows.p, h->dim, h->rank_slot.p, h->nrank, h->dim, h->d_min.p, h->d_inv.p, h->mode,
                PXC_CODE_I8, h->codes.p, h->pitch, s);
  PXC_CUDA(cudaStreamSynchronize(s));
  h->codes_ready = true;
}

// One K12 pass over columns [c_begin, c_end) for nq query rows.
template <int MODE>
void scan_pass(pxc_sq* h, const int8_t* d_q8, uint32_t nq, const uint8_t* d_codes, uint64_t ncodes, uint32_t c_begin,
               uint32_t c_end, uint32_t* dense, uint64_t dense_ld, const uint32_t* tau, uint64_t* cand,
               uint32_t* cnt, uint32_t cap, cudaStream_t s) {
  using namespace sq_tc;
  if (c_end <= c_begin || nq == 0) return;
  const uint32_t kblocks = h->pitch / KB_BYTES;
  const uint32_t stages = pick_stages(kblocks);
  PXC_CONFIG(stages >= 2, "dim", h->dim, "too large for the tensor-core scan");
  const size_t smem = smem_bytes(kblocks, stages);
  PXC_CUDA(cudaFuncSetAttribute(sq_scan_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const uint32_t nq_pad = (uint32_t)round_up(nq, BM);
  CUtensorMap tq, tc;
  make_tmap_u8_2d(&tq, d_q8, h->pitch, nq_pad, KB_BYTES, BM);
  make_tmap_u8_2d(&tc, d_codes, h->pitch, round_up(ncodes, BN), KB_BYTES, BN);
  Params p{};
  p.dense = dense;
  p.dense_ld = dense_ld;
  p.tau = tau;
  p.cand = cand;
  p.cand_cnt = cnt;
  p.cap = cap;
  p.status = h->ctx->d_status;
  p.nq = nq;
  p.c_begin = c_begin;
  p.c_end = c_end;
  p.kblocks = kblocks;
  p.ntiles = (c_end - c_begin + BN - 1) / BN;
  const uint32_t qtiles = nq_pad / BM;
  const uint32_t target = (uint32_t)h->ctx->sm_count * 8;
  uint32_t splits = std::max<uint32_t>(1, std::min<uint32_t>(p.ntiles, (target + qtiles - 1) / qtiles));
  p.tiles_per_split = (p.ntiles + splits - 1) / splits;
  splits = (p.ntiles + p.tiles_per_split - 1) / p.tiles_per_split;
  p.stages = stages;
  p.wait_ns = (uint64_t)h->ctx->wait_ms * 1000000ull;
  sq_scan_kernel<MODE><<<dim3(qtiles, splits), NUM_THREADS, smem, s>>>(tq, tc, p);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 1;
}

uint32_t read_word(pxc_sq* h, const uint32_t* d, cudaStream_t s) {
  PXC_CUDA(cudaMemcpyAsync(h->h_word, d, 4, cudaMemcpyDeviceToHost, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  return *h->h_word;
}

// q8 rows idx[0..n) of the batch into q8s (zero-padded to whole query tiles).
const int8_t* gather_queries(pxc_sq* h, const int8_t* q8, const uint32_t* idx, uint32_t n, cudaStream_t s) {
  const uint32_t pitch = h->pitch;
  const uint32_t n_pad = (uint32_t)round_up(n, sq_tc::BM);
  h->q8s.reserve((size_t)n_pad * pitch);
  PXC_CUDA(cudaMemsetAsync(h->q8s.p, 0, (size_t)n_pad * pitch, s));
  gather_rows16_kernel<<<std::max<uint32_t>(1, std::min<uint32_t>(4096, (n * (pitch / 16) + 255) / 256)), 256, 0, s>>>(
      reinterpret_cast<const uint8_t*>(q8), idx, nullptr, n, pitch, h->q8s.p);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 1;
  return reinterpret_cast<const int8_t*>(h->q8s.p);
}

// The exact fallback for the batch queries in `list` (device, n entries):
// DENSE passes over every column after the prefix, merged chunk by chunk
// into the query's prefix list, which then replaces its final list.
void fallback(pxc_sq* h, const int8_t* q8, const uint32_t* list, uint32_t n, const uint8_t* d_codes, uint64_t nacc,
              uint32_t p0, uint32_t F, cudaStream_t s) {
  const uint32_t n_pad = (uint32_t)round_up(n, sq_tc::BM);
  const int8_t* q8s = gather_queries(h, q8, list, n, s);
  h->Ls.reserve((size_t)n * F);
  h->Ls2.reserve((size_t)n * F);
  h->lens.reserve(n);
  h->lens2.reserve(n);
  gather_lists_kernel<<<n, 256, 0, s>>>(h->L0.p, h->len0.p, list, F, h->Ls.p, h->lens.p);
  h->ctx->launches += 1;
  const uint64_t dcap = (uint64_t)sq::QBATCH * PREFIX;
  const uint32_t chunk = (uint32_t)std::max<uint64_t>(sq_tc::BN, dcap / n_pad / sq_tc::BN * sq_tc::BN);
  uint64_t* La = h->Ls.p;
  uint64_t* Lb = h->Ls2.p;
  uint32_t* la = h->lens.p;
  uint32_t* lb = h->lens2.p;
  for (uint64_t c0 = p0; c0 < nacc; c0 += chunk) {
    const uint32_t c1 = (uint32_t)std::min<uint64_t>(nacc, c0 + chunk);
    const uint64_t ld = round_up(c1 - c0, sq_tc::BN);
    scan_pass<sq_tc::MODE_DENSE>(h, q8s, n, d_codes, nacc, (uint32_t)c0, c1,
                                 h->D.p, ld, nullptr, nullptr, nullptr, 0, s);
    select_chunk_kernel<<<n, SEL_THREADS, 0, s>>>(La, la, Lb, lb, h->D.p, (uint32_t)ld, c0, c1 - (uint32_t)c0, F, 0);
    h->ctx->launches += 1;
    std::swap(La, Lb);
    std::swap(la, lb);
  }
  scatter_lists_kernel<<<n, 256, 0, s>>>(La, la, list, F, h->Lf.p, h->lenf.p);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 1;
}

// One THRESH pass over columns [p0, nacc) for nb query rows, admitting keys
// <= tau[q], then the merge with the prefix lists; failures (overflow, or a
// verification miss when `verify` is given) are listed in fail / n_fail.
void thresh_round(pxc_sq* h, const int8_t* q8, uint32_t nb, const uint8_t* d_codes, uint64_t nacc, uint32_t p0,
                  uint32_t F, uint32_t cap, const uint64_t* L0, const uint32_t* len0, const uint32_t* tau,
                  const uint32_t* verify, const uint32_t* safe_tau, uint64_t* Lout, uint32_t* lenout,
                  uint32_t* next_tau, uint32_t* fail, uint32_t* n_fail, cudaStream_t s) {
  PXC_CUDA(cudaMemsetAsync(h->cnt.p, 0, (size_t)nb * 4, s));
  PXC_CUDA(cudaMemsetAsync(n_fail, 0, 4, s));
  scan_pass<sq_tc::MODE_THRESH>(h, q8, nb, d_codes, nacc, p0, (uint32_t)nacc, nullptr, 0, tau, h->cand.p, h->cnt.p,
                                cap, s);
  merge_kernel<<<nb, 256, CB * 8, s>>>(L0, len0, h->cand.p, h->cnt.p, cap, F, verify, safe_tau, Lout, lenout,
                                       next_tau, fail, n_fail);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 1;
}

void search_device(pxc_sq* h, const float* d_q, uint32_t nq, uint32_t k, uint32_t overfetch, const uint64_t* d_bitmap,
                   const pxc_int_range* ranges, uint32_t nranges, uint64_t* d_ids, float* d_dist, uint32_t* d_len,
                   cudaStream_t s) {
  PXC_CONFIG(h->codes_ready, "index", 0, "the SQ index needs a store and a trained quantizer before search");
  PXC_CONFIG(k <= PXC_MAX_K, "k", k, "exceeds the largest supported k");
  const uint32_t F = std::max(overfetch, k);
  PXC_CONFIG(F <= MAX_OVERFETCH, "overfetch", F, "max(overfetch, k) must be at most 2048");
  PXC_CONFIG(nranges <= MAX_RANGES, "ranges", nranges, "at most 8 range conditions");
  if (nq == 0) return;
  h->timed = false;
  h->last_fallback = 0;
  h->last_retried = 0;
  if (k == 0 || h->nrank == 0) {
    PXC_CUDA(cudaMemsetAsync(d_len, 0, (size_t)nq * 4, s));
    h->last_accepted = 0;
    return;
  }
  const uint32_t pitch = h->pitch;
  // 1. acceptance and compaction
  const uint8_t* d_codes = h->codes.p;
  const uint32_t* acc = nullptr;
  uint64_t nacc = h->nrank;
  if (d_bitmap || nranges) {
    RangeFilter f{};
    f.n = nranges;
    for (uint32_t j = 0; j < nranges; ++j) {
      auto it = h->columns.find(ranges[j].column);
      PXC_CONFIG(it != h->columns.end(), "column", ranges[j].column, "no such metadata column");
      f.values[j] = it->second.first->p;
      f.present[j] = it->second.second ? it->second.second->p : nullptr;
      f.lo[j] = ranges[j].lo;
      f.hi[j] = ranges[j].hi;
    }
    h->flags.reserve(h->nrank);
    h->acc.reserve(h->nrank);
    h->d_nacc.reserve(1);
    const unsigned g = (unsigned)std::min<uint64_t>((h->nrank + 255) / 256, (uint64_t)h->ctx->sm_count * 16);
    accept_kernel<<<g, 256, 0, s>>>(h->rank_slot.p, h->nrank, d_bitmap, f, h->flags.p);
    size_t tmp = 0;
    thrust::counting_iterator<uint32_t> it(0);
    PXC_CUDA(cub::DeviceSelect::Flagged(nullptr, tmp, it, h->flags.p, h->acc.p, h->d_nacc.p, (int64_t)h->nrank, s));
    h->sel_tmp.reserve(std::max<size_t>(tmp, 1));
    PXC_CUDA(cub::DeviceSelect::Flagged(h->sel_tmp.p, tmp, it, h->flags.p, h->acc.p, h->d_nacc.p, (int64_t)h->nrank, s));
    h->ctx->launches += 2;
    nacc = read_word(h, h->d_nacc.p, s);
    if (nacc > 0) {
      const uint64_t rows_pad = round_up(nacc, sq_tc::BN);
      h->codes_c.reserve(rows_pad * pitch);
      PXC_CUDA(cudaMemsetAsync(h->codes_c.p + nacc * pitch, 0, (rows_pad - nacc) * pitch, s));
      const unsigned gg = (unsigned)std::min<uint64_t>((nacc * (pitch / 16) + 255) / 256, (uint64_t)h->ctx->sm_count * 32);
      gather_rows16_kernel<<<gg, 256, 0, s>>>(h->codes.p, h->acc.p, nullptr, nacc, pitch, h->codes_c.p);
      PXC_CUDA(cudaGetLastError());
      h->ctx->launches += 1;
    }
    d_codes = h->codes_c.p;
    acc = h->acc.p;
  }
  h->last_accepted = nacc;
  if (nacc == 0) {
    PXC_CUDA(cudaMemsetAsync(d_len, 0, (size_t)nq * 4, s));
    return;
  }
  // scratch for one batch
  const uint32_t p0 = (uint32_t)std::min<uint64_t>(nacc, PREFIX);
  uint32_t cap = CB - F;
  const uint32_t qb_max = std::min<uint32_t>(nq, QBATCH);
  const uint32_t qb_pad = (uint32_t)round_up(qb_max, sq_tc::BM);
  h->q8.reserve((size_t)qb_pad * pitch);
  h->D.reserve((size_t)QBATCH * PREFIX);
  h->len0.reserve(qb_max);
  h->lenf.reserve(qb_max);
  h->L0.reserve((size_t)qb_max * F);
  h->Lf.reserve((size_t)qb_max * F);
  h->tau.reserve(4 * (size_t)qb_max);  // speculative, safe, gathered next, next
  h->cnt.reserve(qb_max);
  h->ovf.reserve(3 * (size_t)qb_max);  // round-1 failures, round-2 failures, fallback list
  h->n_ovf.reserve(2);
  h->L1.reserve((size_t)qb_max * F);
  h->L2.reserve((size_t)qb_max * F);
  h->len1.reserve(qb_max);
  h->len2.reserve(qb_max);
  if (nacc > p0) h->cand.reserve((size_t)qb_max * cap);
  PXC_CUDA(cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(CB * 8)));
  PXC_CUDA(cudaFuncSetAttribute(rerank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rr_smem(h->dim)));
  PXC_CUDA(cudaFuncSetAttribute(prefix_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(CB * 8)));
  uint32_t cap_limit = 0xFFFFFFFFu;
  {  // diagnostic (pxc_ctx_set_option "sq_candidate_cap"): shrink the THRESH buffers to force the fallback
    const int64_t v = h->ctx->opt_sq_candidate_cap;
    if (v >= 0 && (uint64_t)v < cap) cap = cap_limit = (uint32_t)v;
  }
  if (h->ctx->profiling) {
    if (!h->ev_begin) {
      PXC_CUDA(cudaEventCreate(&h->ev_begin));
      PXC_CUDA(cudaEventCreate(&h->ev_end));
    }
  }
  uint32_t fallback_total = 0, retried_total = 0;
  // speculative admission rank: about SPEC_MARGIN * F of the whole set are expected at or below the
  // r-th key of a p0-column prefix
  uint32_t r_spec = (uint32_t)std::min<uint64_t>(F, std::max<uint64_t>(1, (SPEC_MARGIN * (uint64_t)F * p0 + nacc - 1) / nacc));
  {  // diagnostic (pxc_ctx_set_option "sq_spec_rank"): force the speculative rank
    const int64_t v = h->ctx->opt_sq_spec_rank;
    if (v >= 1 && (uint64_t)v <= F) r_spec = (uint32_t)v;
  }
  for (uint32_t qb = 0; qb < nq; qb += QBATCH) {
    const uint32_t nb = std::min(QBATCH, nq - qb);
    const uint32_t nb_pad = (uint32_t)round_up(nb, sq_tc::BM);
    const float* Qb = d_q + (size_t)qb * h->dim;
    query_s8_kernel<<<nb_pad, 256, 0, s>>>(Qb, nb, h->dim, h->d_scale.p, h->mode == PXC_RANGE_GLOBAL,
                                           reinterpret_cast<int8_t*>(h->q8.p), pitch);
    h->ctx->launches += 1;
    const int8_t* q8 = reinterpret_cast<const int8_t*>(h->q8.p);
    const bool time_it = h->ctx->profiling && nq <= QBATCH;
    if (time_it) PXC_CUDA(cudaEventRecord(h->ev_begin, s));
    // 3a. DENSE prefix and its top-F
    const uint64_t ld0 = round_up(p0, sq_tc::BN);
    scan_pass<sq_tc::MODE_DENSE>(h, q8, nb, d_codes, nacc, 0, p0, h->D.p, ld0, nullptr, nullptr, nullptr, 0, s);
    prefix_select_kernel<<<nb, PSEL_THREADS, CB * 8, s>>>(h->D.p, ld0, p0, F, r_spec, h->L0.p, h->len0.p,
                                                          h->tau.p, h->tau.p + qb_max);
    h->ctx->launches += 1;
    const uint64_t* Lfin = h->L0.p;
    const uint32_t* lfin = h->len0.p;
    if (nacc > p0) {
      // 3b. THRESH over the rest with a speculative admission key (the r-th
      // of the prefix), verified by the merge: a query whose union holds F
      // keys at or below it is exact.
      uint32_t* tau_spec = h->tau.p;
      uint32_t* tau_safe = h->tau.p + qb_max;
      uint32_t* tau_sub = h->tau.p + 2 * (size_t)qb_max;
      uint32_t* tau_next = h->tau.p + 3 * (size_t)qb_max;
      uint32_t* fail1 = h->ovf.p;
      uint32_t* fail2 = h->ovf.p + qb_max;
      uint32_t* fb_list = h->ovf.p + 2 * (size_t)qb_max;
      thresh_round(h, q8, nb, d_codes, nacc, p0, F, cap, h->L0.p, h->len0.p, tau_spec, r_spec < F ? tau_spec : nullptr,
                   tau_safe, h->Lf.p, h->lenf.p, tau_next, fail1, h->n_ovf.p, s);
      const uint32_t n1 = read_word(h, h->n_ovf.p, s);
      retried_total += n1;
      if (n1 > 0) {
        // 3c. the failed queries again with a safe key (F columns are known at or below it), each
        // with the whole candidate buffer shared among them
        const int8_t* q8s = gather_queries(h, q8, fail1, n1, s);
        gather_lists_kernel<<<n1, 256, 0, s>>>(h->L0.p, h->len0.p, fail1, F, h->L1.p, h->len1.p);
        gather_u32_kernel<<<(n1 + 255) / 256, 256, 0, s>>>(tau_next, fail1, n1, tau_sub);
        h->ctx->launches += 2;
        const uint32_t cap2 = (uint32_t)std::min<uint64_t>(0x7FFFFFFFull, (uint64_t)qb_max * (CB - F) / n1);
        thresh_round(h, q8s, n1, d_codes, nacc, p0, F, std::max(cap, std::min<uint32_t>(cap2, cap_limit)), h->L1.p,
                     h->len1.p, tau_sub, nullptr, nullptr, h->L2.p, h->len2.p, nullptr, fail2, h->n_ovf.p + 1, s);
        scatter_lists_kernel<<<n1, 256, 0, s>>>(h->L2.p, h->len2.p, fail1, F, h->Lf.p, h->lenf.p);
        h->ctx->launches += 1;
        const uint32_t n2 = read_word(h, h->n_ovf.p + 1, s);
        if (n2 > 0) {
          // 3d. overflowing buffers: the exact chunked fallback
          gather_u32_kernel<<<(n2 + 255) / 256, 256, 0, s>>>(fail1, fail2, n2, fb_list);
          h->ctx->launches += 1;
          fallback(h, q8, fb_list, n2, d_codes, nacc, p0, F, s);
          fallback_total += n2;
        }
      }
      Lfin = h->Lf.p;
      lfin = h->lenf.p;
    }
    if (time_it) {
      PXC_CUDA(cudaEventRecord(h->ev_end, s));
      h->timed = true;
    }
    // 4. exact re-rank to k
    rerank_kernel<<<nb, RR_THREADS, rr_smem(h->dim), s>>>(Qb, h->dim, Lfin, lfin, F, acc, h->rank_slot.p, h->rows.p, h->ids.p,
                                         h->metric, k, d_ids + (size_t)qb * k, d_dist + (size_t)qb * k, d_len + qb);
    PXC_CUDA(cudaGetLastError());
    h->ctx->launches += 1;
  }
  h->last_fallback = fallback_total;
  h->last_retried = retried_total;
  check_device_status(h->ctx, s, "SQ search (tensor-core scan)");
}

// Store: rows (device, slot order), ids / live on the host.
void set_store(pxc_sq* h, const float* d_rows_or_null, const float* h_rows_or_null, const uint64_t* ids,
               const uint8_t* live, uint64_t nslots, cudaStream_t s) {
  PXC_CONFIG(nslots < 0x7FFFFFFFull, "nslots", nslots, "the device SQ index supports fewer than 2^31 slots");
  std::vector<uint64_t> hid(std::max<uint64_t>(1, nslots));
  for (uint64_t i = 0; i < nslots; ++i) hid[i] = ids ? ids[i] : i;
  if (h_rows_or_null)
    for (uint64_t i = 0; i < nslots * h->dim; ++i)
      if (!std::isfinite(h_rows_or_null[i]))
        throw make_failure(PXC_NON_FINITE, i, 0, "vectors", "vector component %llu is not finite",
                           (unsigned long long)i);
  std::vector<uint32_t> order;
  order.reserve(nslots);
  for (uint64_t i = 0; i < nslots; ++i)
    if (!live || live[i]) order.push_back((uint32_t)i);
  bool sorted = true;
  for (size_t r = 1; r < order.size() && sorted; ++r) sorted = hid[order[r - 1]] < hid[order[r]];
  if (!sorted) std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return hid[a] < hid[b]; });
  for (size_t r = 1; r < order.size(); ++r)
    if (hid[order[r]] == hid[order[r - 1]])
      throw make_failure(PXC_DUPLICATE_ID, hid[order[r]], 0, "ids", "VectorId %llu is live twice",
                         (unsigned long long)hid[order[r]]);
  h->nslots = nslots;
  h->nrank = order.size();
  h->rows.reserve(std::max<uint64_t>(1, nslots * h->dim));
  h->ids.reserve(std::max<uint64_t>(1, nslots));
  h->rank_slot.reserve(std::max<uint64_t>(1, order.size()));
  if (nslots) {
    if (d_rows_or_null)
      PXC_CUDA(cudaMemcpyAsync(h->rows.p, d_rows_or_null, nslots * h->dim * 4, cudaMemcpyDeviceToDevice, s));
    else
      PXC_CUDA(cudaMemcpyAsync(h->rows.p, h_rows_or_null, nslots * h->dim * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(h->ids.p, hid.data(), nslots * 8, cudaMemcpyHostToDevice, s));
  }
  if (!order.empty())
    PXC_CUDA(cudaMemcpyAsync(h->rank_slot.p, order.data(), order.size() * 4, cudaMemcpyHostToDevice, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  for (auto& c : h->columns) {
    delete c.second.first;
    delete c.second.second;
  }
  h->columns.clear();
  h->have_rows = true;
  rebuild_codes(h, s);
}

}  // namespace sq
}  // namespace pxc

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

pxc_status pxc_sq_train(pxc_ctx* ctx, const float* training, uint64_t n, uint32_t dim, int32_t mode, float* out_min,
                        float* out_scale, float* out_inv_scale, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(n > 0 && training, "training", n, "must be a non-empty multiple of the space dimension");
    sq::check_quantizer_args(dim, mode, PXC_CODE_U8);
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = ctx->stream;
    DBuf<float> x;
    x.reserve(n * dim);
    PXC_CUDA(cudaMemcpyAsync(x.p, training, n * dim * 4, cudaMemcpyHostToDevice, s));
    const uint32_t groups = mode == PXC_RANGE_GLOBAL ? 1 : dim;
    std::vector<float> lo(groups), hi(groups);
    sq::ranges_device(ctx, x.p, nullptr, n, dim, mode, lo.data(), hi.data(), s);
    sq::finish_train(groups, lo.data(), hi.data(), out_min, out_scale, out_inv_scale);
  });
}

pxc_status pxc_sq_ranges_device(pxc_ctx* ctx, const float* d_training, uint64_t n, uint32_t dim, int32_t mode,
                                float* out_min, float* out_max, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(n > 0 && d_training, "training", n, "must be a non-empty multiple of the space dimension");
    sq::check_quantizer_args(dim, mode, PXC_CODE_U8);
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    sq::ranges_device(ctx, d_training, nullptr, n, dim, mode, out_min, out_max, s);
  });
}

pxc_status pxc_sq_train_device(pxc_ctx* ctx, const float* d_training, uint64_t n, uint32_t dim, int32_t mode,
                               float* out_min, float* out_scale, float* out_inv_scale, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(n > 0 && d_training, "training", n, "must be a non-empty multiple of the space dimension");
    sq::check_quantizer_args(dim, mode, PXC_CODE_U8);
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    const uint32_t groups = mode == PXC_RANGE_GLOBAL ? 1 : dim;
    std::vector<float> lo(groups), hi(groups);
    sq::ranges_device(ctx, d_training, nullptr, n, dim, mode, lo.data(), hi.data(), s);
    sq::finish_train(groups, lo.data(), hi.data(), out_min, out_scale, out_inv_scale);
  });
}

pxc_status pxc_sq_encode_device(pxc_ctx* ctx, const float* min, const float* inv_scale, uint32_t dim, int32_t mode,
                                int32_t code_type, const float* d_vectors, uint64_t n, uint8_t* d_out_codes,
                                void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    sq::check_quantizer_args(dim, mode, code_type);
    PXC_CONFIG(min && inv_scale, "quantizer", 0, "null range table");
    if (n == 0) return;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    const uint32_t groups = mode == PXC_RANGE_GLOBAL ? 1 : dim;
    DBuf<float> t;
    t.reserve(2 * groups);
    PXC_CUDA(cudaMemcpyAsync(t.p, min, groups * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(t.p + groups, inv_scale, groups * 4, cudaMemcpyHostToDevice, s));
    sq::encode_device(ctx, d_vectors, dim, nullptr, n, dim, t.p, t.p + groups, mode, code_type, d_out_codes, dim, s);
    PXC_CUDA(cudaStreamSynchronize(s));
  });
}

pxc_status pxc_sq_encode(pxc_ctx* ctx, const float* min, const float* inv_scale, uint32_t dim, int32_t mode,
                         int32_t code_type, const float* vectors, uint64_t n, uint8_t* out_codes, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    sq::check_quantizer_args(dim, mode, code_type);
    PXC_CONFIG(min && inv_scale, "quantizer", 0, "null range table");
    if (n == 0) return;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = ctx->stream;
    const uint32_t groups = mode == PXC_RANGE_GLOBAL ? 1 : dim;
    DBuf<float> t, x;
    DBuf<uint8_t> c;
    t.reserve(2 * groups);
    x.reserve(n * dim);
    c.reserve(n * dim);
    PXC_CUDA(cudaMemcpyAsync(t.p, min, groups * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(t.p + groups, inv_scale, groups * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(x.p, vectors, n * dim * 4, cudaMemcpyHostToDevice, s));
    sq::encode_device(ctx, x.p, dim, nullptr, n, dim, t.p, t.p + groups, mode, code_type, c.p, dim, s);
    PXC_CUDA(cudaMemcpyAsync(out_codes, c.p, n * dim, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
  });
}

pxc_status pxc_sq_decode(pxc_ctx* ctx, const float* min, const float* scale, uint32_t dim, int32_t mode,
                         int32_t code_type, const uint8_t* codes, uint64_t n, float* out, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    sq::check_quantizer_args(dim, mode, code_type);
    PXC_CONFIG(min && scale, "quantizer", 0, "null range table");
    if (n == 0) return;
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = ctx->stream;
    const uint32_t groups = mode == PXC_RANGE_GLOBAL ? 1 : dim;
    DBuf<float> t, x;
    DBuf<uint8_t> c;
    t.reserve(2 * groups);
    x.reserve(n * dim);
    c.reserve(n * dim);
    PXC_CUDA(cudaMemcpyAsync(t.p, min, groups * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(t.p + groups, scale, groups * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(c.p, codes, n * dim, cudaMemcpyHostToDevice, s));
    const unsigned blocks = (unsigned)std::min<uint64_t>((n * dim + 255) / 256, (uint64_t)ctx->sm_count * 32);
    sq::decode_kernel<<<blocks, 256, 0, s>>>(c.p, n, dim, t.p, t.p + groups, mode == PXC_RANGE_GLOBAL,
                                             code_type == PXC_CODE_I8, x.p);
    PXC_CUDA(cudaGetLastError());
    ctx->launches += 1;
    PXC_CUDA(cudaMemcpyAsync(out, x.p, n * dim * 4, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
  });
}

pxc_status pxc_sq_asymmetric_device(pxc_ctx* ctx, const float* min, const float* scale, uint32_t dim, int32_t mode,
                                    int32_t code_type, int32_t metric, const float* d_queries, uint32_t nq,
                                    const uint8_t* d_codes, uint64_t n, float* d_out, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    sq::check_quantizer_args(dim, mode, code_type);
    PXC_CONFIG(min && scale, "quantizer", 0, "null range table");
    PXC_CONFIG(metric == PXC_EUCLIDEAN || metric == PXC_INNER_PRODUCT || metric == PXC_COSINE, "metric", metric,
               "asymmetric scoring is squared L2 (euclidean) or the negated dot (inner product, cosine)");
    PXC_CONFIG(nq <= 65535u * sq::ASYM_Q, "nq", nq, "at most 524280 queries per call");
    if (nq == 0 || n == 0) return;
    PXC_CONFIG(d_queries && d_codes && d_out, "buffers", 0, "null buffer");
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    const uint32_t groups = mode == PXC_RANGE_GLOBAL ? 1 : dim;
    DBuf<float> t;
    t.reserve(2 * groups);
    PXC_CUDA(cudaMemcpyAsync(t.p, min, groups * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(t.p + groups, scale, groups * 4, cudaMemcpyHostToDevice, s));
    const dim3 grid((unsigned)((n + 127) / 128), (nq + sq::ASYM_Q - 1) / sq::ASYM_Q);
    sq::asymmetric_kernel<<<grid, 128, 0, s>>>(d_queries, nq, d_codes, n, dim, t.p, t.p + groups,
                                               mode == PXC_RANGE_GLOBAL, code_type == PXC_CODE_I8,
                                               metric != PXC_EUCLIDEAN, d_out);
    PXC_CUDA(cudaGetLastError());
    ctx->launches += 1;
    PXC_CUDA(cudaStreamSynchronize(s));  // the range table is freed on return
  });
}

pxc_status pxc_sq_asymmetric(pxc_ctx* ctx, const float* min, const float* scale, uint32_t dim, int32_t mode,
                             int32_t code_type, int32_t metric, const float* queries, uint32_t nq,
                             const uint8_t* codes, uint64_t n, float* out, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    sq::check_quantizer_args(dim, mode, code_type);
    if (nq == 0 || n == 0) return;
    PXC_CONFIG(queries && codes && out, "buffers", 0, "null buffer");
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = ctx->stream;
    DBuf<float> dq, dout;
    DBuf<uint8_t> dc;
    dq.reserve((size_t)nq * dim);
    dc.reserve(n * dim);
    dout.reserve((size_t)nq * n);
    PXC_CUDA(cudaMemcpyAsync(dq.p, queries, (size_t)nq * dim * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(dc.p, codes, n * dim, cudaMemcpyHostToDevice, s));
    pxc_error e2{};
    if (pxc_sq_asymmetric_device(ctx, min, scale, dim, mode, code_type, metric, dq.p, nq, dc.p, n, dout.p, s, &e2) !=
        PXC_OK)
      throw make_failure((pxc_status)e2.code, e2.a, e2.b, e2.parameter, "%s", e2.detail);
    PXC_CUDA(cudaMemcpyAsync(out, dout.p, (size_t)nq * n * 4, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
  });
}

pxc_status pxc_sq_create(pxc_ctx* ctx, uint32_t dim, int32_t metric, pxc_sq** out, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr && out != nullptr, "ctx", 0, "null argument");
    PXC_CONFIG(dim > 0 && dim <= sq::MAX_DIM, "dim", dim, "the SQ index supports 1 <= dim <= 1024");
    PXC_CONFIG(metric == PXC_COSINE || metric == PXC_INNER_PRODUCT, "metric", metric,
               "the SQ index scores cosine and inner product");
    DeviceGuard g(ctx->device);
    auto* h = new pxc_sq();
    h->ctx = ctx;
    h->dim = dim;
    h->pitch = (uint32_t)sq::round_up(dim, sq_tc::KB_BYTES);
    h->metric = metric;
    cudaError_t e = cudaMallocHost(&h->h_word, 16);
    if (e != cudaSuccess) {
      delete h;
      PXC_CUDA(e);
    }
    *out = h;
  });
}

void pxc_sq_destroy(pxc_sq* h) {
  if (!h) return;
  DeviceGuard g(h->ctx->device);
  delete h;
}

pxc_status pxc_sq_set_quantizer(pxc_sq* h, int32_t mode, const float* min, const float* scale, const float* inv_scale,
                                pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    sq::check_quantizer_args(h->dim, mode, PXC_CODE_I8);
    PXC_CONFIG(min && scale && inv_scale, "quantizer", 0, "null range table");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = h->ctx->stream;
    const uint32_t groups = mode == PXC_RANGE_GLOBAL ? 1 : h->dim;
    h->mode = mode;
    h->h_min.assign(min, min + groups);
    h->h_scale.assign(scale, scale + groups);
    h->h_inv.assign(inv_scale, inv_scale + groups);
    h->d_min.reserve(groups);
    h->d_scale.reserve(groups);
    h->d_inv.reserve(groups);
    PXC_CUDA(cudaMemcpyAsync(h->d_min.p, min, groups * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(h->d_scale.p, scale, groups * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(h->d_inv.p, inv_scale, groups * 4, cudaMemcpyHostToDevice, s));
    h->have_quantizer = true;
    sq::rebuild_codes(h, s);
  });
}

pxc_status pxc_sq_get_quantizer(pxc_sq* h, int32_t* mode, float* min, float* scale, float* inv_scale, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr && h->have_quantizer, "h", 0, "no quantizer");
    std::lock_guard<std::mutex> lock(h->mu);
    if (mode) *mode = h->mode;
    if (min) std::copy(h->h_min.begin(), h->h_min.end(), min);
    if (scale) std::copy(h->h_scale.begin(), h->h_scale.end(), scale);
    if (inv_scale) std::copy(h->h_inv.begin(), h->h_inv.end(), inv_scale);
  });
}

pxc_status pxc_sq_train_store(pxc_sq* h, int32_t mode, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr && h->have_rows, "h", 0, "the SQ index has no store");
    sq::check_quantizer_args(h->dim, mode, PXC_CODE_I8);
    PXC_CONFIG(h->nrank > 0, "training", 0, "must be a non-empty multiple of the space dimension");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = h->ctx->stream;
    const uint32_t groups = mode == PXC_RANGE_GLOBAL ? 1 : h->dim;
    std::vector<float> lo(groups), hi(groups), mn(groups), sc(groups), inv(groups);
    if (h->nrank == h->nslots) {
      sq::ranges_device(h->ctx, h->rows.p, nullptr, h->nslots, h->dim, mode, lo.data(), hi.data(), s);
    } else {
      // live rows only, in slot order
      std::vector<uint32_t> rs(h->nrank);
      PXC_CUDA(cudaMemcpyAsync(rs.data(), h->rank_slot.p, h->nrank * 4, cudaMemcpyDeviceToHost, s));
      PXC_CUDA(cudaStreamSynchronize(s));
      std::sort(rs.begin(), rs.end());
      DBuf<uint32_t> map;
      map.reserve(h->nrank);
      PXC_CUDA(cudaMemcpyAsync(map.p, rs.data(), h->nrank * 4, cudaMemcpyHostToDevice, s));
      sq::ranges_device(h->ctx, h->rows.p, map.p, h->nrank, h->dim, mode, lo.data(), hi.data(), s);
    }
    sq::finish_train(groups, lo.data(), hi.data(), mn.data(), sc.data(), inv.data());
    h->mode = mode;
    h->h_min = mn;
    h->h_scale = sc;
    h->h_inv = inv;
    h->d_min.reserve(groups);
    h->d_scale.reserve(groups);
    h->d_inv.reserve(groups);
    PXC_CUDA(cudaMemcpyAsync(h->d_min.p, mn.data(), groups * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(h->d_scale.p, sc.data(), groups * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(h->d_inv.p, inv.data(), groups * 4, cudaMemcpyHostToDevice, s));
    h->have_quantizer = true;
    sq::rebuild_codes(h, s);
  });
}

pxc_status pxc_sq_set_store(pxc_sq* h, const float* vectors, const uint64_t* ids, const uint8_t* live, uint64_t nslots,
                            pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    PXC_CONFIG(nslots == 0 || vectors, "vectors", 0, "null vectors");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    sq::set_store(h, nullptr, vectors, ids, live, nslots, h->ctx->stream);
  });
}

pxc_status pxc_sq_set_store_device(pxc_sq* h, const float* d_vectors, const uint64_t* ids, const uint8_t* live,
                                   uint64_t nslots, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    PXC_CONFIG(nslots == 0 || d_vectors, "vectors", 0, "null vectors");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    sq::set_store(h, d_vectors, nullptr, ids, live, nslots, h->ctx->stream);
  });
}

pxc_status pxc_sq_set_column(pxc_sq* h, uint32_t column, const int64_t* values, const uint8_t* present,
                             pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr && h->have_rows, "h", 0, "the SQ index has no store");
    PXC_CONFIG(h->nslots == 0 || values, "values", 0, "null values");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = h->ctx->stream;
    auto& slot = h->columns[column];
    if (!slot.first) slot.first = new DBuf<int64_t>();
    slot.first->reserve(std::max<uint64_t>(1, h->nslots));
    if (h->nslots) PXC_CUDA(cudaMemcpyAsync(slot.first->p, values, h->nslots * 8, cudaMemcpyHostToDevice, s));
    delete slot.second;
    slot.second = nullptr;
    if (present) {
      slot.second = new DBuf<uint8_t>();
      slot.second->reserve(std::max<uint64_t>(1, h->nslots));
      if (h->nslots) PXC_CUDA(cudaMemcpyAsync(slot.second->p, present, h->nslots, cudaMemcpyHostToDevice, s));
    }
    PXC_CUDA(cudaStreamSynchronize(s));
  });
}

uint64_t pxc_sq_len(const pxc_sq* h) { return h ? h->nrank : 0; }

pxc_status pxc_sq_get_codes(pxc_sq* h, uint8_t* out_codes, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr && h->codes_ready, "h", 0, "no codes (store and quantizer needed)");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = h->ctx->stream;
    std::vector<uint8_t> rc(h->nrank * h->pitch);
    std::vector<uint32_t> rs(h->nrank);
    if (h->nrank) {
      PXC_CUDA(cudaMemcpyAsync(rc.data(), h->codes.p, rc.size(), cudaMemcpyDeviceToHost, s));
      PXC_CUDA(cudaMemcpyAsync(rs.data(), h->rank_slot.p, h->nrank * 4, cudaMemcpyDeviceToHost, s));
    }
    PXC_CUDA(cudaStreamSynchronize(s));
    std::memset(out_codes, 0, h->nslots * h->dim);
    for (uint64_t r = 0; r < h->nrank; ++r)
      std::memcpy(out_codes + (uint64_t)rs[r] * h->dim, rc.data() + r * h->pitch, h->dim);
  });
}

pxc_status pxc_sq_search_device(pxc_sq* h, const float* d_queries, uint32_t nq, uint32_t k, uint32_t overfetch,
                                const uint64_t* d_bitmap, const pxc_int_range* ranges, uint32_t nranges,
                                uint64_t* d_out_ids, float* d_out_dist, uint32_t* d_out_len, void* stream,
                                pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    PXC_CONFIG(nranges == 0 || ranges, "ranges", nranges, "null range array");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->ctx->stream;
    sq::search_device(h, d_queries, nq, k, overfetch, d_bitmap, ranges, nranges, d_out_ids, d_out_dist, d_out_len, s);
  });
}

pxc_status pxc_sq_search(pxc_sq* h, const float* queries, uint32_t nq, uint32_t k, uint32_t overfetch,
                         const uint64_t* bitmap, const pxc_int_range* ranges, uint32_t nranges, uint64_t* out_ids,
                         float* out_dist, uint32_t* out_len, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    PXC_CONFIG(nranges == 0 || ranges, "ranges", nranges, "null range array");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = h->ctx->stream;
    if (nq == 0) return;
    for (uint64_t i = 0; i < (uint64_t)nq * h->dim; ++i)
      if (!std::isfinite(queries[i]))
        throw make_failure(PXC_NON_FINITE, i % h->dim, 0, "query", "query component %llu is not finite",
                           (unsigned long long)(i % h->dim));
    const size_t kk = std::max<uint32_t>(k, 1);
    h->q_dev.reserve((size_t)nq * h->dim);
    h->o_ids.reserve((size_t)nq * kk);
    h->o_dist.reserve((size_t)nq * kk);
    h->o_len.reserve(nq);
    DBuf<uint64_t> bm;
    if (bitmap) {
      const uint64_t words = (h->nslots + 63) / 64;
      bm.reserve(std::max<uint64_t>(1, words));
      if (words) PXC_CUDA(cudaMemcpyAsync(bm.p, bitmap, words * 8, cudaMemcpyHostToDevice, s));
    }
    PXC_CUDA(cudaMemcpyAsync(h->q_dev.p, queries, (size_t)nq * h->dim * 4, cudaMemcpyHostToDevice, s));
    sq::search_device(h, h->q_dev.p, nq, k, overfetch, bitmap ? bm.p : nullptr, ranges, nranges, h->o_ids.p,
                      h->o_dist.p, h->o_len.p, s);
    if (k) {
      PXC_CUDA(cudaMemcpyAsync(out_ids, h->o_ids.p, (size_t)nq * k * 8, cudaMemcpyDeviceToHost, s));
      PXC_CUDA(cudaMemcpyAsync(out_dist, h->o_dist.p, (size_t)nq * k * 4, cudaMemcpyDeviceToHost, s));
    }
    PXC_CUDA(cudaMemcpyAsync(out_len, h->o_len.p, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
  });
}

float pxc_sq_last_scan_ms(pxc_sq* h) {
  if (!h || !h->timed) return -1.0f;
  float ms = -1.0f;
  if (cudaEventSynchronize(h->ev_end) != cudaSuccess) return -1.0f;
  if (cudaEventElapsedTime(&ms, h->ev_begin, h->ev_end) != cudaSuccess) return -1.0f;
  return ms;
}

uint64_t pxc_sq_last_accepted(const pxc_sq* h) { return h ? h->last_accepted : 0; }
uint32_t pxc_sq_last_fallback(const pxc_sq* h) { return h ? h->last_fallback : 0; }
uint32_t pxc_sq_last_retried(const pxc_sq* h) { return h ? h->last_retried : 0; }

}  // extern "C"
