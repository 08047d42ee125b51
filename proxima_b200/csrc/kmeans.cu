// kmeans.cu — Lloyd's k-means on the device, equal to the reference's
// `kmeans` (crates/proxima-quantize/src/kmeans.rs:59-143) bit for bit on a
// single GPU: the same assignments, f64 sums, centroids, inertia and
// iteration count from the same initial centroids.
//
// Per iteration:
//   assignment  exact = argmin over centroids of the sequential f32 sum
//               sum_d (p_d - c_d)^2 (kmeans.rs:200-212, 234-241), ties to the
//               lower index. Two ways, same answer:
//                 * K7 exact path: CUDA cores evaluate that sum for every
//                   (point, centroid) pair in the reference's order;
//                 * K7 screened path (dim 16..128, k >= 256): tensor cores
//                   (K7a, kmeans_tc.cuh) bound every centroid's score, only the
//                   centroids that can still win are evaluated exactly, and a
//                   point whose screen is inconclusive is rescanned exactly.
//   inertia     the sequential f64 sum of the winners' distances (seqsum.cuh).
//   update      K8: points are stably sorted by cluster; one warp per cluster
//               sums its members in ascending point order in f64 and writes
//               (sum * (1/count)) as f32 — the reference's order exactly.
//               Empty clusters are re-seeded in index order at the farthest
//               point against the partially updated centroids (exact, with
//               distance bounds that limit the exact scans to the few points
//               that can be the farthest).
// Seeding: the injected initial centroids, or k-means++ (K9) with ChaCha8.
#include <cub/cub.cuh>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <vector>

#include "common.cuh"
#include "kmeans_api.h"
#include "kmeans_tc.cuh"
#include "rng.h"
#include "seqsum.cuh"
#include "tmap.cuh"

namespace pxc {
namespace km {

constexpr uint32_t INVALID = 0xFFFFFFFFu;
constexpr int TC = 64;  // centroids per shared-memory tile (tiled exact kernel)
constexpr uint32_t MAX_DIM = 512;
constexpr uint32_t SEEDS = 32;  // about this many best-bounded points are scanned first when re-seeding
constexpr uint32_t SCREEN_FALLBACK = 16384;  // more candidates than this: tighten the bounds by screening

// squared (kmeans.rs:234-241): sequential, no fused multiply-add.
__device__ __forceinline__ float seq_l2(const float* __restrict__ a, const float* __restrict__ b, uint32_t d) {
  float s = 0.0f;
#pragma unroll 4
  for (uint32_t i = 0; i < d; ++i) {
    const float t = __fsub_rn(__ldg(a + i), __ldg(b + i));
    s = __fadd_rn(s, __fmul_rn(t, t));
  }
  return s;
}

// Each lane gets the distance between A row ia and B row ib: the warp stages
// its 32 row pairs through shared memory 32 dimensions at a time with
// coalesced 16-byte loads (row pitches are multiples of 4 floats, bases
// 16-byte aligned), and each lane continues its own sums over the staged
// chunk. U8 = false: one sequential sum (kmeans.rs `squared`); U8 = true:
// eight lane sums over full chunks of 8, reduced pairwise, plus a sequential
// tail (proxima_core::distance::squared_euclidean).
// sa, sb: 32 x 33 floats each, private to the warp.
template <bool U8>
__device__ __forceinline__ float warp_rows_l2(const float* __restrict__ A, uint32_t lda, uint64_t ia,
                                              const float* __restrict__ B, uint32_t ldb, uint64_t ib, uint32_t d,
                                              float* sa, float* sb) {
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t part = lane & 7;  // which 4 dimensions of the 32-wide chunk
  const uint32_t full = d & ~7u;
  float s = 0.0f, tail = 0.0f;
  float acc[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) acc[l] = 0.0f;
  for (uint32_t c0 = 0; c0 < d; c0 += 32) {
    const bool on = c0 + part * 4 < d;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int row = q * 4 + (int)(lane >> 3);
      const uint64_t ra = __shfl_sync(0xFFFFFFFFu, ia, row);
      const uint64_t rb = __shfl_sync(0xFFFFFFFFu, ib, row);
      float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f), y = x;
      if (on) {
        x = __ldg(reinterpret_cast<const float4*>(A + ra * lda + c0) + part);
        y = __ldg(reinterpret_cast<const float4*>(B + rb * ldb + c0) + part);
      }
      float* pa = sa + row * 33 + part * 4;
      float* pb = sb + row * 33 + part * 4;
      pa[0] = x.x, pa[1] = x.y, pa[2] = x.z, pa[3] = x.w;
      pb[0] = y.x, pb[1] = y.y, pb[2] = y.z, pb[3] = y.w;
    }
    __syncwarp();
    const uint32_t cnt = min(32u, d - c0);
    if (U8) {
      const uint32_t vfull = c0 + 32 <= full ? 32u : (full > c0 ? full - c0 : 0u);
      for (uint32_t j = 0; j < vfull; j += 8) {
#pragma unroll
        for (int l = 0; l < 8; ++l) {
          const float t = __fsub_rn(sa[lane * 33 + j + l], sb[lane * 33 + j + l]);
          acc[l] = __fadd_rn(acc[l], __fmul_rn(t, t));
        }
      }
      for (uint32_t j = vfull; j < cnt; ++j) {
        const float t = __fsub_rn(sa[lane * 33 + j], sb[lane * 33 + j]);
        tail = __fadd_rn(tail, __fmul_rn(t, t));
      }
    } else {
      for (uint32_t j = 0; j < cnt; ++j) {
        const float t = __fsub_rn(sa[lane * 33 + j], sb[lane * 33 + j]);
        s = __fadd_rn(s, __fmul_rn(t, t));
      }
    }
    __syncwarp();
  }
  if (U8) {
    const float x = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
    const float y = __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7]));
    return __fadd_rn(__fadd_rn(x, y), tail);
  }
  return s;
}

// ---------------------------------------------------------------------------
// K7 exact, tiled: a block of PB points (transposed into shared memory)
// against 64-centroid tiles; each thread keeps eight running sums, one per
// centroid of a group, and walks the dimensions in order.
// Optional `list`: the points to assign, count in *list_count.
// mode 1: write assign (setting *changed when it moves) and bestd;
// mode 0: write bestd only.
// ---------------------------------------------------------------------------
template <bool U8>
__global__ void __launch_bounds__(128) assign_exact_kernel(
    const float* __restrict__ P, uint32_t ldp, uint64_t n, const uint32_t* __restrict__ list,
    const uint32_t* __restrict__ list_count, const float* __restrict__ C, uint32_t ldc, uint32_t k, uint32_t d,
    uint32_t csplit, unsigned long long* __restrict__ keys, uint32_t* __restrict__ assign,
    float* __restrict__ bestd, uint32_t* __restrict__ changed, int mode, uint32_t* __restrict__ ver,
    uint32_t ver_val) {
  extern __shared__ __align__(16) float sm[];
  const uint32_t PB = blockDim.x, PBS = PB + 1;
  float* ps = sm;                                        // [d][PBS]
  float* cs = sm + (((size_t)d * PBS + 3) & ~size_t(3));  // [d][TC]
  __shared__ uint32_t rows[128];
  const uint64_t nl = list ? (uint64_t)*list_count : n;
  const uint64_t row0 = (uint64_t)blockIdx.x * PB;
  if (row0 >= nl) return;
  const uint32_t t = threadIdx.x;
  const uint32_t pi = row0 + t < nl ? (list ? list[row0 + t] : (uint32_t)(row0 + t)) : INVALID;
  rows[t] = pi;
  __syncthreads();
  for (uint32_t e = t; e < PB * d; e += PB) {
    const uint32_t r = e / d, i = e - r * d;
    const uint32_t q = rows[r];
    ps[i * PBS + r] = q != INVALID ? P[(size_t)q * ldp + i] : 0.0f;
  }
  float best = __int_as_float(0x7f800000);
  uint32_t bi = 0;
  const uint32_t cbeg = blockIdx.y * csplit, cend = min(k, cbeg + csplit);
  for (uint32_t c0 = cbeg; c0 < cend; c0 += TC) {
    const uint32_t cnt = min((uint32_t)TC, cend - c0);
    __syncthreads();
    for (uint32_t e = t; e < TC * d; e += PB) {
      const uint32_t j = e / d, i = e - j * d;
      cs[i * TC + j] = j < cnt ? C[(size_t)(c0 + j) * ldc + i] : 0.0f;
    }
    __syncthreads();
    if (U8) {  // one centroid at a time, eight lane sums
      const uint32_t full = d & ~7u;
      for (uint32_t j = 0; j < cnt; ++j) {
        float acc[8];
#pragma unroll
        for (int l = 0; l < 8; ++l) acc[l] = 0.0f;
        for (uint32_t i = 0; i < full; i += 8) {
#pragma unroll
          for (int l = 0; l < 8; ++l) {
            const float df = __fsub_rn(ps[(i + l) * PBS + t], cs[(i + l) * TC + j]);
            acc[l] = __fadd_rn(acc[l], __fmul_rn(df, df));
          }
        }
        float tail = 0.0f;
        for (uint32_t i = full; i < d; ++i) {
          const float df = __fsub_rn(ps[i * PBS + t], cs[i * TC + j]);
          tail = __fadd_rn(tail, __fmul_rn(df, df));
        }
        const float x = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
        const float y = __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7]));
        const float D = __fadd_rn(__fadd_rn(x, y), tail);
        if (D < best) {
          best = D;
          bi = c0 + j;
        }
      }
      continue;
    }
    for (uint32_t g = 0; g < cnt; g += 8) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
#pragma unroll 2
      for (uint32_t i = 0; i < d; ++i) {
        const float pv = ps[i * PBS + t];
        const float4 a = *reinterpret_cast<const float4*>(cs + i * TC + g);
        const float4 b = *reinterpret_cast<const float4*>(cs + i * TC + g + 4);
        const float cv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float df = __fsub_rn(pv, cv[j]);
          acc[j] = __fadd_rn(acc[j], __fmul_rn(df, df));
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (g + j < cnt && acc[j] < best) {
          best = acc[j];
          bi = c0 + g + j;
        }
    }
  }
  if (pi == INVALID) return;
  if (keys) {  // one of several centroid ranges: (distance, index) minimum
    atomicMin(keys + pi, ((unsigned long long)__float_as_uint(best) << 32) | bi);
    return;
  }
  if (mode == 1 && assign[pi] != bi) *changed = 1u;
  if (mode >= 1) assign[pi] = bi;
  if (ver) ver[pi] = ver_val;
  bestd[pi] = best;
}

// Resolves the (distance, index) keys of a centroid-split exact scan.
__global__ void resolve_keys_kernel(const uint32_t* __restrict__ list, const uint32_t* __restrict__ count,
                                    unsigned long long* __restrict__ keys, uint32_t* __restrict__ assign,
                                    float* __restrict__ bestd, uint32_t* __restrict__ changed, int mode,
                                    uint32_t* __restrict__ ver, uint32_t ver_val) {
  const uint32_t nl = *count;
  for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < nl; j += gridDim.x * blockDim.x) {
    const uint32_t pi = list[j];
    const unsigned long long kk = keys[pi];
    keys[pi] = ~0ull;
    const uint32_t bi = (uint32_t)kk;
    if (mode == 1 && assign[pi] != bi) *changed = 1u;
    if (mode >= 1) assign[pi] = bi;
    if (ver) ver[pi] = ver_val;
    bestd[pi] = __uint_as_float((uint32_t)(kk >> 32));
  }
}

// Squared norms in fp32 (any order: only used for bounds and the screened
// scores), +inf for rows in [rows, pad_to); the largest finite one as bits.
__global__ void sqnorm_kernel(const float* __restrict__ X, uint32_t ld, uint64_t rows, uint32_t d,
                              uint64_t pad_to, float* __restrict__ out, uint32_t* __restrict__ maxbits) {
  const uint64_t warp = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const uint32_t lane = threadIdx.x & 31;
  if (warp >= pad_to) return;
  if (warp >= rows) {
    if (lane == 0) out[warp] = __int_as_float(0x7f800000);
    return;
  }
  float s = 0.0f;
  for (uint32_t i = lane; i < d; i += 32) {
    const float v = X[warp * ld + i];
    s = fmaf(v, v, s);
  }
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  if (lane == 0) {
    out[warp] = s;
    if (maxbits) atomicMax(maxbits, __float_as_uint(s));
  }
}

// out[i] = distance(P row i, C row idx[i]) for every point (warp-cooperative).
template <bool U8>
__global__ void __launch_bounds__(128) pair_l2_kernel(const float* __restrict__ P, uint32_t ldp, uint64_t n, uint32_t d,
                                                      const float* __restrict__ C, uint32_t ldc,
                                                      const uint32_t* __restrict__ idx, float* __restrict__ out) {
  __shared__ float stage[4][2][32 * 33];
  const uint32_t w = threadIdx.x >> 5;
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  const bool valid = i < n;
  const float s = warp_rows_l2<U8>(P, ldp, valid ? i : 0, C, ldc, valid ? idx[i] : 0, d, stage[w][0], stage[w][1]);
  if (valid) out[i] = s;
}

// Per-point bounds for the screening kernel. Every centroid able to win (or
// tie) the exact argmin has a screened score a(c) = ||c||^2 - 2 p.c below
//   T = U/(1-gamma) - ||p||^2_lo + E
// for any U that bounds the winner's exact distance from above, where
//   u        f32 unit roundoff 2^-24
//   gamma    relative error of the reference's sequential distance, (d+4)u
//   E        bound on |a_screened(c) - a(c)|: TF32 operands lose at most 2^-10
//            relative each and FP32 accumulation adds less than d*2^-22, so
//            |dot error| < 2^-8 ||p|| ||c||; plus the FP32 norm (2(d+1)u ||c||^2),
//            the rounding of the score itself, and flushed tiny operands.
// Two such U: the exact distance to some centroid (`exact`, giving T_prior),
// and, from the smallest screened score m, (1+gamma)(||p||^2_hi + m + E),
// which gives T(m) = A (B + m) + Cc with A = (1+gamma)/(1-gamma),
// B = ||p||^2_hi + E and Cc = E - ||p||^2_lo. All are rounded up.
__host__ __device__ inline double screen_gamma(uint32_t d) { return (d + 4) * 0x1p-24 * 1.01; }

__global__ void bound_kernel(uint64_t n, uint32_t d, const float* __restrict__ pnorm,
                             const uint32_t* __restrict__ cmax_bits, const float* __restrict__ exact,
                             const float* __restrict__ amin, float4* __restrict__ out) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const double u = 0x1p-24, et = 0x1p-8;
  const double gam = screen_gamma(d);
  const double rel = (d + 2) * u * 1.01;
  const double pn = pnorm[i];
  const double pn_hi = pn * (1.0 + rel), pn_lo = fmax(0.0, pn * (1.0 - rel));
  const double cm = (double)__uint_as_float(*cmax_bits) * (1.0 + rel);
  const double pr = sqrt(pn_hi) * (1.0 + 1e-12), cr = sqrt(cm) * (1.0 + 1e-12);
  const double E = 2.0 * et * pr * cr + 2.0 * (d + 1) * u * cm + 4.0 * u * (cm + 2.0 * pr * cr) + d * 0x1p-75;
  float4 o;
  if (exact || amin) {
    const double U = exact ? (double)exact[i] : (1.0 + gam) * fmax(0.0, pn_hi + (double)amin[i] + E);
    double T = U / (1.0 - gam) - pn_lo + E;
    T += fabs(T) * 0x1p-40 + 1e-37;
    o.x = __double2float_ru(T);
  } else {
    o.x = __int_as_float(0x7f800000);
  }
  o.y = __double2float_ru(pn_hi + E);
  o.z = __double2float_ru(E - pn_lo);
  o.w = 0.0f;
  out[i] = o;
}

// Exact re-scoring of the screened candidates, warp-cooperative (ascending
// centroid order per point; '<' with the index tie-break keeps the lower
// index). Inconclusive points (no candidate, or more than CMAX) go to the
// rescan list.
template <bool U8>
__global__ void __launch_bounds__(128) cand_eval_kernel(const float* __restrict__ P, uint32_t ldp, uint64_t n,
                                                        uint32_t d, const float* __restrict__ C, uint32_t ldc, uint32_t k,
                                                        const uint32_t* __restrict__ cnt,
                                                        const uint32_t* __restrict__ cand, uint32_t* __restrict__ assign,
                                                        float* __restrict__ bestd, uint32_t* changed,
                                                        uint32_t* __restrict__ rescan, uint32_t* rescan_count,
                                                        int mode) {
  __shared__ float stage[4][2][32 * 33];
  const uint32_t w = threadIdx.x >> 5;
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  const bool valid = i < n;
  const uint32_t c_n = valid ? cnt[i] : 0u;
  const uint32_t m = (c_n >= 1 && c_n <= (uint32_t)km_tc::CMAX) ? c_n : 0u;
  const uint32_t mmax = __reduce_max_sync(0xFFFFFFFFu, m);
  float best = __int_as_float(0x7f800000);
  uint32_t bi = INVALID;
  for (uint32_t j = 0; j < mmax; ++j) {
    const uint32_t c = j < m ? cand[i * km_tc::CMAX + j] : INVALID;
    const float D = warp_rows_l2<U8>(P, ldp, valid ? i : 0, C, ldc, c < k ? c : 0u, d, stage[w][0], stage[w][1]);
    if (c < k && (D < best || (D == best && c < bi))) {
      best = D;
      bi = c;
    }
  }
  if (!valid) return;
  if (bi == INVALID) {
    rescan[atomicAdd(rescan_count, 1u)] = (uint32_t)i;
    return;
  }
  if (mode == 1) {
    if (assign[i] != bi) *changed = 1u;
    assign[i] = bi;
  }
  bestd[i] = best;
}

// K8: cluster boundaries in the (cluster, point)-sorted order.
__global__ void offsets_kernel(const uint32_t* __restrict__ keys, uint64_t n, uint32_t k, uint32_t* __restrict__ off) {
  const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c > k) return;
  uint64_t lo = 0, hi = n;
  while (lo < hi) {
    const uint64_t mid = (lo + hi) >> 1;
    if (keys[mid] < c)
      lo = mid + 1;
    else
      hi = mid;
  }
  off[c] = (uint32_t)lo;
}

// K8: one warp per (cluster, group of 32 dimensions), lanes over dimensions;
// members in ascending point order, f64 running sums from 0.0, then
// (sum * (1.0/count)) as f32 (kmeans.rs:104-135). Each lane's sum is its own
// sequential chain, so splitting dimensions across warps keeps the order.
// Empty clusters are counted (once) and left for the re-seed.
__global__ void cluster_mean_kernel(const float* __restrict__ P, uint32_t ldp, uint32_t d, uint32_t groups,
                                    const uint32_t* __restrict__ sorted, const uint32_t* __restrict__ off, uint32_t k,
                                    float* __restrict__ out, uint32_t ldc, uint32_t* empty_count) {
  const uint32_t w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t c = w / groups, g = w - c * groups;
  if (c >= k) return;
  const uint32_t b = off[c], e = off[c + 1];
  if (b == e) {
    if (lane == 0 && g == 0) atomicAdd(empty_count, 1u);
    return;
  }
  const uint32_t dim = g * 32 + lane;
  const bool on = dim < d;
  const float* base = P + dim;
  double s = 0.0;
  for (uint32_t m0 = b; m0 < e; m0 += 32) {
    const uint32_t cntm = min(32u, e - m0);
    const uint32_t mine = lane < cntm ? sorted[m0 + lane] : 0u;
    uint32_t j = 0;
    for (; j + 8 <= cntm; j += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint32_t pt = __shfl_sync(0xFFFFFFFFu, mine, j + u);
        v[u] = on ? __ldg(base + (size_t)pt * ldp) : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) s = __dadd_rn(s, (double)v[u]);
    }
    for (; j < cntm; ++j) {
      const uint32_t pt = __shfl_sync(0xFFFFFFFFu, mine, j);
      const float v = on ? __ldg(base + (size_t)pt * ldp) : 0.0f;
      s = __dadd_rn(s, (double)v);
    }
  }
  if (on) out[(size_t)c * ldc + dim] = __double2float_rn(__dmul_rn(s, 1.0 / (double)(e - b)));
}

// Point-sharded update, this rank's half: per cluster the f64 sums of the
// rank's members in point order (the chains of cluster_mean_kernel) and the
// member count; empty clusters write zeros.
__global__ void cluster_sum_kernel(const float* __restrict__ P, uint32_t ldp, uint32_t d, uint32_t groups,
                                   const uint32_t* __restrict__ sorted, const uint32_t* __restrict__ off, uint32_t k,
                                   double* __restrict__ sums, uint32_t* __restrict__ counts) {
  const uint32_t w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t c = w / groups, g = w - c * groups;
  if (c >= k) return;
  const uint32_t b = off[c], e = off[c + 1];
  const uint32_t dim = g * 32 + lane;
  const bool on = dim < d;
  if (lane == 0 && g == 0) counts[c] = e - b;
  const float* base = P + dim;
  double s = 0.0;
  for (uint32_t m0 = b; m0 < e; m0 += 32) {
    const uint32_t cntm = min(32u, e - m0);
    const uint32_t mine = lane < cntm ? sorted[m0 + lane] : 0u;
    for (uint32_t j = 0; j < cntm; ++j) {
      const uint32_t pt = __shfl_sync(0xFFFFFFFFu, mine, j);
      const float v = on ? __ldg(base + (size_t)pt * ldp) : 0.0f;
      s = __dadd_rn(s, (double)v);
    }
  }
  if (on) sums[(size_t)c * d + dim] = s;
}

// The other half: every rank's sums folded in rank order (the ranks hold
// consecutive ranges of the point order), the counts added, and
// c = (sum * (1.0/count)) as f32 (kmeans.rs:127-135). Segment of rank r at
// all + r * seg: sums [k][d] f64, then counts [k] u32. gcount: the global counts.
__global__ void fold_means_kernel(const unsigned char* __restrict__ all, size_t seg, uint32_t nranks, uint32_t k,
                                  uint32_t d, float* __restrict__ next, uint32_t ldc, uint32_t* __restrict__ gcount,
                                  uint32_t* __restrict__ empty_count) {
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (uint64_t)k * d) return;
  const uint32_t c = (uint32_t)(t / d), j = (uint32_t)(t - (uint64_t)c * d);
  double S = 0.0;
  uint32_t N = 0;
  for (uint32_t r = 0; r < nranks; ++r) {
    const double* sums = reinterpret_cast<const double*>(all + r * seg);
    const uint32_t* cnt = reinterpret_cast<const uint32_t*>(all + r * seg + (size_t)k * d * 8);
    S = __dadd_rn(S, sums[(size_t)c * d + j]);
    N += cnt[c];
  }
  if (j == 0) gcount[c] = N;
  if (N == 0) {
    if (j == 0) atomicAdd(empty_count, 1u);
    return;
  }
  next[(size_t)c * ldc + j] = __double2float_rn(__dmul_rn(S, 1.0 / (double)N));
}

// Sharded re-seeding: this rank's farthest point (a key of argmax_list_kernel)
// as a segment [key u64, global index u64, the point's d floats].
__global__ void farthest_candidate_kernel(const float* __restrict__ P, uint32_t ldp, uint32_t d,
                                          const unsigned long long* __restrict__ key, uint64_t global_first,
                                          unsigned char* __restrict__ seg) {
  const unsigned long long kk = *key;
  const uint64_t idx = 0xFFFFFFFFull - (kk & 0xFFFFFFFFull);
  if (threadIdx.x == 0) {
    reinterpret_cast<unsigned long long*>(seg)[0] = kk;
    reinterpret_cast<unsigned long long*>(seg)[1] = global_first + idx;
  }
  float* row = reinterpret_cast<float*>(seg + 16);
  for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) row[i] = P[idx * ldp + i];
}
// The global farthest point among the ranks' candidates: the largest
// distance, ties to the lowest global index (farthest_point's strict '>'
// over the whole point order), copied into the centroid row.
__global__ void farthest_pick_kernel(const unsigned char* __restrict__ all, size_t seg, uint32_t nranks, uint32_t d,
                                     float* __restrict__ dst) {
  __shared__ uint32_t best;
  if (threadIdx.x == 0) {
    uint32_t b = 0;
    for (uint32_t r = 1; r < nranks; ++r) {
      const unsigned long long* kr = reinterpret_cast<const unsigned long long*>(all + r * seg);
      const unsigned long long* kb = reinterpret_cast<const unsigned long long*>(all + b * seg);
      const uint32_t dr = (uint32_t)(kr[0] >> 32), db = (uint32_t)(kb[0] >> 32);
      if (dr > db || (dr == db && kr[1] < kb[1])) b = r;
    }
    best = b;
  }
  __syncthreads();
  const float* row = reinterpret_cast<const float*>(all + best * seg + 16);
  for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) dst[i] = row[i];
}

// farthest_point (kmeans.rs:215-226) helpers: largest distance, first index on
// ties, as one u64 key (distance bits, then the complemented index).
__global__ void argmax_list_kernel(const float* __restrict__ v, const uint32_t* __restrict__ list,
                                   const uint32_t* __restrict__ count_ptr, uint32_t count_val,
                                   unsigned long long* key) {
  unsigned long long best = 0;
  const uint32_t nl = count_ptr ? *count_ptr : count_val;
  for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < nl; j += gridDim.x * blockDim.x) {
    const uint32_t i = list[j];
    const unsigned long long kk = ((unsigned long long)__float_as_uint(v[i]) << 32) | (0xFFFFFFFFull - i);
    best = kk > best ? kk : best;
  }
  for (int o = 16; o; o >>= 1) {
    const unsigned long long x = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    best = x > best ? x : best;
  }
  if ((threadIdx.x & 31) == 0) atomicMax(key, best);
}

// Copies point row `index` (from a key of argmax_list_kernel) into a centroid row.
__global__ void copy_row_kernel(const float* __restrict__ P, uint32_t ldp, uint32_t d,
                                const unsigned long long* __restrict__ key, float* __restrict__ dst) {
  const uint64_t idx = 0xFFFFFFFFull - (*key & 0xFFFFFFFFull);
  for (uint32_t i = threadIdx.x; i < d; i += blockDim.x) dst[i] = P[idx * ldp + i];
}

// Re-seeding bounds. Each point keeps ub (an upper bound on its nearest
// distance in the current centroid set), ubc (the centroid row it was measured
// against) and ube (the empty cluster being processed when it was measured;
// rows below that index were then in their updated version). When rows
// [ube, e) have switched to their updated version since, the bound is
// re-measured against the row as it now stands (for the point's own cluster
// that distance, u_next, is precomputed).
constexpr uint32_t UB_SCREENED = 0xFFFFFFFEu;  // ubc of a bound from a screening pass

__device__ __forceinline__ float ub_refresh(const float* __restrict__ P, uint32_t ldp, uint64_t i, uint32_t d,
                                            const float* __restrict__ next, uint32_t ldc,
                                            const uint32_t* __restrict__ assign, const float* __restrict__ u_next,
                                            const float* __restrict__ u_cur, uint32_t e, float* __restrict__ ub,
                                            uint32_t* __restrict__ ubc, uint32_t* __restrict__ ube) {
  const uint32_t c = ubc[i];
  if (c == UB_SCREENED) {  // a screened bound holds for its own set only
    if (ube[i] == e) return ub[i];
    const uint32_t a = assign[i];
    const float v = a < e ? u_next[i] : u_cur[i];
    ub[i] = v;
    ubc[i] = a;
    ube[i] = e;
    return v;
  }
  if (c < ube[i] || c >= e) return ub[i];
  const float v = c == assign[i] ? u_next[i] : seq_l2(P + i * ldp, next + (size_t)c * ldc, d);
  ub[i] = v;
  ube[i] = e;
  return v;
}

// Refreshes the bounds and histograms them for choosing seeds: the points in
// the top bins of a 2048-bin histogram of the bounds (bits >> 20 of a
// non-negative float: exponent and three mantissa bits), about `want` of
// them, at most `cap`.
__global__ void ub_hist_kernel(const float* __restrict__ P, uint32_t ldp, uint64_t n, uint32_t d,
                               const float* __restrict__ next, uint32_t ldc, const uint32_t* __restrict__ assign,
                               const float* __restrict__ u_next, const float* __restrict__ u_cur, uint32_t e,
                               float* __restrict__ ub,
                               uint32_t* __restrict__ ubc, uint32_t* __restrict__ ube, uint32_t* __restrict__ hist) {
  __shared__ uint32_t h[2048];
  for (uint32_t b = threadIdx.x; b < 2048; b += blockDim.x) h[b] = 0;
  __syncthreads();
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const float v = ub_refresh(P, ldp, i, d, next, ldc, assign, u_next, u_cur, e, ub, ubc, ube);
    atomicAdd(&h[__float_as_uint(v) >> 20], 1u);
  }
  __syncthreads();
  for (uint32_t b = threadIdx.x; b < 2048; b += blockDim.x)
    if (h[b]) atomicAdd(hist + b, h[b]);
}
// The bin, counted from the top of a 2048-bin histogram, where the top
// `want` entries end: *bin, and the count of entries in bins above it. One
// block of 256 threads, eight bins each, suffix sums by a block scan.
__device__ void top_bin(const uint32_t* __restrict__ h, uint32_t want, uint32_t* bin, uint32_t* above) {
  using Scan = cub::BlockScan<uint32_t, 256>;
  __shared__ typename Scan::TempStorage tmp;
  const uint32_t t = threadIdx.x;
  uint32_t c[8], sum = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {  // thread t owns bins 2047-8t down to 2040-8t
    c[j] = h[2047 - 8 * t - j];
    sum += c[j];
  }
  uint32_t before;  // entries in the bins above this thread's
  Scan(tmp).ExclusiveSum(sum, before);
  if (t == 0) {
    *bin = 0;
    *above = before;  // overwritten below unless want exceeds everything
  }
  __syncthreads();
  if (before < want && before + sum >= want) {
    uint32_t acc = before;
    for (int j = 0; j < 8; ++j) {
      if (acc + c[j] >= want) {
        *bin = 2047 - 8 * t - j;
        *above = acc;
        break;
      }
      acc += c[j];
    }
  }
}

// tau[0] = first-level bin b1, tau[1] = entries above it.
__global__ void __launch_bounds__(256) ub_level1_kernel(const uint32_t* __restrict__ hist, uint32_t want,
                                                        uint32_t* tau) {
  top_bin(hist, want, tau, tau + 1);
}
// Second level: bin b1 histogrammed again on the next 11 bits.
__global__ void ub_hist2_kernel(const float* __restrict__ ub, uint64_t n, uint32_t* __restrict__ hist,
                                const uint32_t* __restrict__ tau) {
  __shared__ uint32_t h[2048];
  const uint32_t b1 = tau[0];
  for (uint32_t b = threadIdx.x; b < 2048; b += blockDim.x) h[b] = 0;
  __syncthreads();
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t bits = __float_as_uint(ub[i]);
    if ((bits >> 20) == b1) atomicAdd(&h[(bits >> 9) & 2047u], 1u);
  }
  __syncthreads();
  for (uint32_t b = threadIdx.x; b < 2048; b += blockDim.x)
    if (h[b]) atomicAdd(hist + 2048 + b, h[b]);
}
// tau[2] = the threshold bits for the top `want` bounds.
__global__ void __launch_bounds__(256) ub_level2_kernel(const uint32_t* __restrict__ hist, uint32_t want,
                                                        uint32_t* tau) {
  __shared__ uint32_t b2, above2;
  const uint32_t left = want > tau[1] ? want - tau[1] : 1u;
  top_bin(hist + 2048, left, &b2, &above2);
  __syncthreads();
  if (threadIdx.x == 0) tau[2] = (tau[0] << 20) | (b2 << 9);
}

// Gathers the points whose bound reaches the threshold (ties included, at
// most `cap`).
__global__ void ub_gather_kernel(const float* __restrict__ ub, uint64_t n, const uint32_t* __restrict__ tau,
                                 uint32_t cap, uint32_t* __restrict__ list, uint32_t* count) {
  const uint32_t t = tau[2];
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    if (__float_as_uint(ub[i]) >= t) {
      const uint32_t pos = atomicAdd(count, 1u);
      if (pos < cap) list[pos] = (uint32_t)i;
    }
}
__global__ void clamp_count_kernel(uint32_t* count, uint32_t cap) {
  if (*count > cap) *count = cap;
}

// Tightens the bounds with a screening (MIN) pass over the current set: the
// nearest exact distance is at most (1+gamma)(||p||^2_hi + m + E), m the
// smallest screened score (see bound_kernel).
__global__ void ub_screened_kernel(uint64_t n, uint32_t d, const float* __restrict__ pnorm,
                                   const uint32_t* __restrict__ cmax_bits, const float* __restrict__ amin, uint32_t e,
                                   float* __restrict__ ub, uint32_t* __restrict__ ubc, uint32_t* __restrict__ ube) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const double u = 0x1p-24, et = 0x1p-8;
  const double gam = (d + 4) * u * 1.01, rel = (d + 2) * u * 1.01;
  const double pn_hi = (double)pnorm[i] * (1.0 + rel);
  const double cm = (double)__uint_as_float(*cmax_bits) * (1.0 + rel);
  const double pr = sqrt(pn_hi) * (1.0 + 1e-12), cr = sqrt(cm) * (1.0 + 1e-12);
  const double E = 2.0 * et * pr * cr + 2.0 * (d + 1) * u * cm + 4.0 * u * (cm + 2.0 * pr * cr) + d * 0x1p-75;
  double U = (1.0 + gam) * fmax(0.0, pn_hi + (double)amin[i] + E);
  U += U * 0x1p-40 + 1e-37;
  const float v = __double2float_ru(U);
  if (v < ub[i]) {
    ub[i] = v;
    ubc[i] = UB_SCREENED;
    ube[i] = e;
  }
}

// Points that can still be the farthest: ub >= the best exact distance found
// among the seeds (key: argmax_list_kernel over the seeds).
__global__ void ub_filter_kernel(const float* __restrict__ ub, uint64_t n, const unsigned long long* __restrict__ key,
                                 uint32_t* list, uint32_t* count) {
  const float lb = __uint_as_float((uint32_t)(*key >> 32));
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    if (ub[i] >= lb) list[atomicAdd(count, 1u)] = (uint32_t)i;
}

// K9 (kmeans.rs:156-159, 182-189): nearest_sq against a new centre, strict '<'.
__global__ void __launch_bounds__(128) kpp_update_kernel(const float* __restrict__ P, uint32_t ldp, uint64_t n,
                                                         uint32_t d, const float* __restrict__ c,
                                                         float* __restrict__ nearest, int first) {
  extern __shared__ __align__(16) float sm[];
  const uint32_t PB = blockDim.x, PBS = PB + 1;
  float* ps = sm;  // [d][PBS]
  float* cs = sm + (((size_t)d * PBS + 3) & ~size_t(3));
  const uint64_t row0 = (uint64_t)blockIdx.x * PB;
  const uint32_t t = threadIdx.x;
  for (uint32_t e = t; e < PB * d; e += PB) {
    const uint32_t r = e / d, i = e - r * d;
    ps[i * PBS + r] = row0 + r < n ? P[(row0 + r) * ldp + i] : 0.0f;
  }
  for (uint32_t i = t; i < d; i += PB) cs[i] = c[i];
  __syncthreads();
  if (row0 + t >= n) return;
  float s = 0.0f;
  for (uint32_t i = 0; i < d; ++i) {
    const float df = __fsub_rn(ps[i * PBS + t], cs[i]);
    s = __fadd_rn(s, __fmul_rn(df, df));
  }
  if (first || s < nearest[row0 + t]) nearest[row0 + t] = s;
}

// Validation: first non-finite element (as a flat index) and the largest |x|.
__global__ void scan_input_kernel(const float* __restrict__ P, uint32_t ldp, uint64_t n, uint32_t d,
                                  unsigned long long* first_bad, uint32_t* maxabs) {
  uint32_t m = 0;
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t w0 = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const uint64_t nw = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  for (uint64_t r = w0; r < n; r += nw)
    for (uint32_t i = lane; i < d; i += 32) {
      const uint32_t b = __float_as_uint(P[r * ldp + i]) & 0x7FFFFFFFu;
      if (b >= 0x7F800000u)
        atomicMin(first_bad, (unsigned long long)(r * d + i));
      else
        m = max(m, b);
    }
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  if (lane == 0) atomicMax(maxabs, m);
}

// Trace only: histogram of screened candidate counts (0, 1, ..., 8, more).
__global__ void cand_hist_kernel(const uint32_t* __restrict__ cnt, uint64_t n, uint32_t* hist) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    atomicAdd(hist + min(cnt[i], 9u), 1u);
}

__global__ void iota_kernel(uint32_t* out, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    out[i] = (uint32_t)i;
}

// ---------------------------------------------------------------------------
// Host driver
// ---------------------------------------------------------------------------

// Scratch kept on the context between calls: device buffers only grow, and
// the pinned host words are allocated once.
struct Workspace {
  DBuf<float> cur, next, part, cnorm, pnorm, bestd, u_next, exact, amin, nearest, ub;
  DBuf<float4> bound;
  DBuf<uint32_t> assign, cnt, cand, rescan, keys_a, keys_b, iota, sorted, off, words, ubc, ube, hist;
  DBuf<unsigned long long> key, keys;
  DBuf<unsigned char> sort_tmp;
  uint64_t iota_n = 0, keys_n = 0;
  uint32_t* h_words = nullptr;          // pinned: [0] changed [1] list count [2] empty count
  double* h_double = nullptr;           // pinned
  unsigned long long* h_u64 = nullptr;  // pinned: [0] pick, [1..2] validation scratch
  seqsum::Summer summer;
  cudaEvent_t prof[2] = {};
  ~Workspace() {
    for (cudaEvent_t e : prof)
      if (e) cudaEventDestroy(e);
    if (h_words) cudaFreeHost(h_words);
    if (h_double) cudaFreeHost(h_double);
    if (h_u64) cudaFreeHost(h_u64);
  }
  static void destroy(void* p) { delete static_cast<Workspace*>(p); }
};

Workspace& workspace(pxc_ctx* ctx) {
  if (!ctx->kmeans_ws) {
    ctx->kmeans_ws = new Workspace();
    ctx->kmeans_ws_free = &Workspace::destroy;
  }
  Workspace& w = *static_cast<Workspace*>(ctx->kmeans_ws);
  if (!w.h_words) PXC_CUDA(cudaMallocHost(&w.h_words, 8 * sizeof(uint32_t)));
  if (!w.h_double) PXC_CUDA(cudaMallocHost(&w.h_double, 2 * sizeof(double)));
  if (!w.h_u64) PXC_CUDA(cudaMallocHost(&w.h_u64, 4 * sizeof(unsigned long long)));
  return w;
}

struct Runner {
  pxc_ctx* ctx = nullptr;
  cudaStream_t s = nullptr;
  const float* P = nullptr;  // device, pitch ldp
  uint32_t ldp = 0;
  uint64_t n = 0;
  uint32_t d = 0, k = 0, ldc = 0;
  bool tensor = false;
  bool trace = false;
  bool unrolled = false;  // exact distances in squared_euclidean's 8-lane order
  uint64_t launches = 0;

  Workspace& w;
  DBuf<float>&cur, &next, &part, &cnorm, &pnorm, &bestd, &u_next, &exact, &amin, &nearest, &ub;
  DBuf<float4>& bound;
  DBuf<uint32_t>&assign, &cnt, &cand, &rescan, &keys_a, &keys_b, &iota, &sorted, &off, &words, &ubc, &ube, &hist;
  DBuf<unsigned long long>&key, &keys;
  DBuf<unsigned char>& sort_tmp;
  size_t sort_tmp_bytes = 0;
  uint32_t* h_words;
  double* h_double;
  unsigned long long* h_u64;
  seqsum::Summer& summer;
  cudaEvent_t* prof;

  explicit Runner(Workspace& ws)
      : w(ws), cur(ws.cur), next(ws.next), part(ws.part), cnorm(ws.cnorm), pnorm(ws.pnorm), bestd(ws.bestd),
        u_next(ws.u_next), exact(ws.exact), amin(ws.amin), nearest(ws.nearest), ub(ws.ub), bound(ws.bound),
        assign(ws.assign), cnt(ws.cnt), cand(ws.cand), rescan(ws.rescan), keys_a(ws.keys_a), keys_b(ws.keys_b),
        iota(ws.iota), sorted(ws.sorted), off(ws.off), words(ws.words), ubc(ws.ubc), ube(ws.ube), hist(ws.hist),
        key(ws.key), keys(ws.keys), sort_tmp(ws.sort_tmp), h_words(ws.h_words), h_double(ws.h_double),
        h_u64(ws.h_u64), summer(ws.summer), prof(ws.prof) {}
  CUtensorMap tmap_p;
  uint32_t kblocks = 0, stages = 0, ntiles = 0;
  // Point-sharded mode (pxc_kmeans_sharded): this rank holds points
  // [global_first, global_first + n) of the global order; the per-iteration
  // state is exchanged over the context's communicator.
  bool sharded = false;
  uint64_t global_first = 0;
  DBuf<unsigned char> xs, xr;
  DBuf<uint32_t> gcount;
  std::vector<uint32_t> h_gcount;

  cudaEvent_t ev[8] = {};
  uint32_t screen_passes = 0;
  float screen_ms = 0.0f;
  void mark(int i) {
    if (!trace) return;
    if (!ev[i]) PXC_CUDA(cudaEventCreate(&ev[i]));
    PXC_CUDA(cudaEventRecord(ev[i], s));
  }
  float span(int a, int b) {
    float ms = 0.0f;
    PXC_CUDA(cudaEventSynchronize(ev[b]));
    PXC_CUDA(cudaEventElapsedTime(&ms, ev[a], ev[b]));
    return ms;
  }

  ~Runner() {
    for (cudaEvent_t e : ev)
      if (e) cudaEventDestroy(e);
  }

  uint32_t exact_block() const { return d <= 128 ? 128 : (d <= 256 ? 64 : 32); }
  size_t exact_smem(uint32_t pb) const {
    return ((((size_t)d * (pb + 1) + 3) & ~size_t(3)) + (size_t)d * TC) * sizeof(float);
  }
  unsigned blocks(uint64_t threads, uint32_t per) const { return (unsigned)((threads + per - 1) / per); }

  void setup(bool want_tensor) {
    const uint64_t kpad = ((uint64_t)k + km_tc::BN - 1) / km_tc::BN * km_tc::BN;
    for (DBuf<float>* b : {&cur, &next, &part}) {
      b->reserve((size_t)kpad * ldc);
      PXC_CUDA(cudaMemsetAsync(b->p, 0, (size_t)kpad * ldc * 4, s));
    }
    cnorm.reserve(kpad);
    for (DBuf<float>* b : {&pnorm, &bestd, &u_next, &exact, &ub}) b->reserve(n);
    for (DBuf<uint32_t>* b : {&assign, &rescan, &keys_a, &keys_b, &iota, &sorted, &ubc, &ube}) b->reserve(n);
    hist.reserve(4096 + 4);
    off.reserve((size_t)k + 1);
    words.reserve(8);
    key.reserve(2);
    if (w.keys_n < n) {  // (distance, index) keys start at ~0 and are reset after each use
      keys.reserve(n);
      PXC_CUDA(cudaMemsetAsync(keys.p, 0xFF, n * 8, s));
      w.keys_n = n;
    }
    PXC_CUDA(cudaMemsetAsync(assign.p, 0, n * 4, s));
    size_t need = 0, need2 = 0;
    PXC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, need, keys_a.p, keys_b.p, iota.p, sorted.p, (int)n, 0, 32, s));
    PXC_CUDA(cub::DeviceRadixSort::SortPairsDescending(nullptr, need2, keys_a.p, keys_b.p, iota.p, sorted.p, (int)n,
                                                       0, 32, s));
    sort_tmp_bytes = std::max(need, need2);
    sort_tmp.reserve(sort_tmp_bytes);
    if (w.iota_n < n) {
      iota_kernel<<<ctx->sm_count * 4, 256, 0, s>>>(iota.p, n);
      ++launches;
      w.iota_n = n;
    }
    tensor = want_tensor;
    if (ctx->profiling)
      for (int i = 0; i < 2; ++i)
        if (!prof[i]) PXC_CUDA(cudaEventCreate(&prof[i]));
    if (tensor) {
      kblocks = (d + km_tc::KB_FLOATS - 1) / km_tc::KB_FLOATS;
      stages = km_tc::pick_stages(kblocks);
      ntiles = (uint32_t)(kpad / km_tc::BN);
      bound.reserve(n);
      amin.reserve(n);
      cnt.reserve(n);
      cand.reserve(n * km_tc::CMAX);
      make_tmap_f32_2d(&tmap_p, P, d, ldp, n, km_tc::KB_FLOATS, km_tc::BM);
      const size_t smem = km_tc::smem_bytes(kblocks, stages);
      PXC_CUDA(cudaFuncSetAttribute(km_tc::screen_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      PXC_CUDA(cudaFuncSetAttribute(km_tc::screen_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      sqnorm_kernel<<<blocks(n * 32, 256), 256, 0, s>>>(P, ldp, n, d, n, pnorm.p, nullptr);
      ++launches;
    }
    const uint32_t pb = exact_block();
    PXC_CUDA(cudaFuncSetAttribute(assign_exact_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)exact_smem(pb)));
    PXC_CUDA(cudaFuncSetAttribute(assign_exact_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)exact_smem(pb)));
    PXC_CUDA(cudaFuncSetAttribute(kpp_update_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)exact_smem(pb)));
  }

  // Exact nearest centroid for the points listed in `list` (count on the
  // device at *dcount, `nl` on the host): the tiled kernel over a 2-D grid of
  // point blocks x centroid ranges, so that short lists still fill the GPU.
  void exact_list(const float* C, const uint32_t* list, const uint32_t* dcount, uint32_t nl, uint32_t* asg,
                  float* bd, int mode, uint32_t* ver = nullptr, uint32_t ver_val = 0) {
    if (nl == 0) return;
    const uint32_t pb = exact_block();
    const uint32_t gx = blocks(nl, pb);
    const uint32_t tiles = (k + TC - 1) / TC;
    const uint32_t want = std::max<uint32_t>(1, (2u * ctx->sm_count + gx - 1) / gx);
    const uint32_t splits = std::min(tiles, want);
    const uint32_t csplit = (tiles + splits - 1) / splits * TC;
    const uint32_t gy = (k + csplit - 1) / csplit;
    auto kern = unrolled ? assign_exact_kernel<true> : assign_exact_kernel<false>;
    if (gy == 1) {
      kern<<<dim3(gx, 1), pb, exact_smem(pb), s>>>(P, ldp, n, list, dcount, C, ldc, k, d, csplit, nullptr, asg, bd,
                                                   words.p + 0, mode, ver, ver_val);
      ++launches;
    } else {
      kern<<<dim3(gx, gy), pb, exact_smem(pb), s>>>(P, ldp, n, list, dcount, C, ldc, k, d, csplit, keys.p, asg, bd,
                                                    words.p + 0, mode, nullptr, 0);
      resolve_keys_kernel<<<std::min<uint32_t>(blocks(nl, 256), ctx->sm_count * 8), 256, 0, s>>>(
          list, dcount, keys.p, asg, bd, words.p + 0, mode, ver, ver_val);
      launches += 2;
    }
    PXC_CUDA(cudaGetLastError());
  }

  uint32_t read_word(int i) {
    PXC_CUDA(cudaMemcpyAsync(h_words + i, words.p + i, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    return h_words[i];
  }

  // Screening-kernel parameters for centroid set C (norms already in cnorm,
  // the largest in words[4]).
  km_tc::Params screen_params(const float* C, CUtensorMap* tmap_c) {
    make_tmap_f32_2d(tmap_c, C, d, ldc, k, km_tc::KB_FLOATS, km_tc::BN);
    km_tc::Params prm{};
    prm.cnorm = cnorm.p;
    prm.bound = bound.p;
    prm.A = (float)((1.0 + screen_gamma(d)) / (1.0 - screen_gamma(d)) * (1.0 + 0x1p-30));
    prm.out_min = amin.p;
    prm.out_cnt = cnt.p;
    prm.out_cand = cand.p;
    prm.status = ctx->d_status;
    prm.npoints = (uint32_t)n;
    prm.kblocks = kblocks;
    prm.ntiles = ntiles;
    prm.stages = stages;
    prm.wait_ns = (uint64_t)ctx->wait_ms * 1000000ull;
    return prm;
  }

  // MIN screening pass against C: amin = smallest screened score per point.
  void screen(const float* C, bool) {
    CUtensorMap tmap_c;
    const km_tc::Params prm = screen_params(C, &tmap_c);
    km_tc::screen_kernel<true><<<blocks(n, km_tc::BM), km_tc::NUM_THREADS, km_tc::smem_bytes(kblocks, stages), s>>>(
        tmap_p, tmap_c, prm);
    ++launches;
    PXC_CUDA(cudaGetLastError());
  }

  // Assignment pass against centroids `C` (k rows): writes assign (+ changed
  // in words[0]) and bestd. `prior`: the current assignment's exact distances
  // bound the winners (not on the first pass).
  void nearest_pass(const float* C, bool prior, uint64_t* rescanned) {
    PXC_CUDA(cudaMemsetAsync(words.p, 0, 8 * sizeof(uint32_t), s));
    if (!tensor) {
      const uint32_t pb = exact_block();
      auto kern = unrolled ? assign_exact_kernel<true> : assign_exact_kernel<false>;
      kern<<<blocks(n, pb), pb, exact_smem(pb), s>>>(P, ldp, n, nullptr, nullptr, C, ldc, k, d, k, nullptr, assign.p,
                                                     bestd.p, words.p + 0, 1, nullptr, 0);
      ++launches;
      PXC_CUDA(cudaGetLastError());
      return;
    }
    const uint64_t kpad = (uint64_t)ntiles * km_tc::BN;
    sqnorm_kernel<<<blocks(kpad * 32, 256), 256, 0, s>>>(C, ldc, k, d, kpad, cnorm.p, words.p + 4);
    CUtensorMap tmap_c;
    const km_tc::Params prm = screen_params(C, &tmap_c);
    const unsigned grid = blocks(n, km_tc::BM);
    const size_t smem = km_tc::smem_bytes(kblocks, stages);
    mark(0);
    if (prior) {
      (unrolled ? pair_l2_kernel<true> : pair_l2_kernel<false>)<<<blocks(n, 128), 128, 0, s>>>(P, ldp, n, d, C, ldc,
                                                                                              assign.p, exact.p);
      bound_kernel<<<blocks(n, 256), 256, 0, s>>>(n, d, pnorm.p, words.p + 4, exact.p, nullptr, bound.p);
    } else {
      km_tc::screen_kernel<true><<<grid, km_tc::NUM_THREADS, smem, s>>>(tmap_p, tmap_c, prm);
      bound_kernel<<<blocks(n, 256), 256, 0, s>>>(n, d, pnorm.p, words.p + 4, nullptr, amin.p, bound.p);
    }
    mark(6);
    if (ctx->profiling) PXC_CUDA(cudaEventRecord(prof[0], s));
    km_tc::screen_kernel<false><<<grid, km_tc::NUM_THREADS, smem, s>>>(tmap_p, tmap_c, prm);
    if (ctx->profiling) PXC_CUDA(cudaEventRecord(prof[1], s));
    mark(1);
    (unrolled ? cand_eval_kernel<true> : cand_eval_kernel<false>)<<<blocks(n, 128), 128, 0, s>>>(
        P, ldp, n, d, C, ldc, k, cnt.p, cand.p, assign.p, bestd.p, words.p + 0, rescan.p, words.p + 1, 1);
    launches += 4;
    PXC_CUDA(cudaGetLastError());
    PXC_CUDA(cudaMemcpyAsync(ctx->h_status, ctx->d_status, 2 * sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    const uint32_t nres = read_word(1);
    if (ctx->h_status[0]) check_device_status(ctx, s, "k-means screening");
    ++screen_passes;
    if (ctx->profiling) {
      float ms = 0.0f;
      PXC_CUDA(cudaEventElapsedTime(&ms, prof[0], prof[1]));
      screen_ms += ms;
    }
    if (trace) {
      DBuf<uint32_t> hist;
      hist.reserve(10);
      uint32_t h[10];
      PXC_CUDA(cudaMemsetAsync(hist.p, 0, sizeof(h), s));
      cand_hist_kernel<<<ctx->sm_count * 4, 256, 0, s>>>(cnt.p, n, hist.p);
      PXC_CUDA(cudaMemcpyAsync(h, hist.p, sizeof(h), cudaMemcpyDeviceToHost, s));
      PXC_CUDA(cudaStreamSynchronize(s));
      std::fprintf(stderr, "[pxc kmeans] pass prior=%d bound=%.3f ms screen=%.3f ms rescans=%u candidates:",
                   (int)prior, span(0, 6), span(6, 1), nres);
      for (int b = 0; b < 10; ++b) std::fprintf(stderr, " %u", h[b]);
      std::fprintf(stderr, "\n");
    }
    exact_list(C, rescan.p, words.p + 1, nres, assign.p, bestd.p, 1);
    if (rescanned) *rescanned += nres;
  }

  double seq_sum(const float* v, bool keep_prefix) {
    launches += summer.enqueue(v, n, keep_prefix, s, ctx->sm_count);
    PXC_CUDA(cudaMemcpyAsync(h_double, summer.result.p, sizeof(double), cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    return h_double[0];
  }

  // k-means++ (kmeans.rs:146-194) into cur.
  void seed_kpp(ChaCha8& rng) {
    const uint32_t pb = exact_block();
    nearest.reserve(n);
    const uint64_t first = rng.gen_index(n);
    PXC_CUDA(cudaMemcpyAsync(cur.p, P + first * ldp, d * sizeof(float), cudaMemcpyDeviceToDevice, s));
    kpp_update_kernel<<<blocks(n, pb), pb, exact_smem(pb), s>>>(P, ldp, n, d, cur.p, nearest.p, 1);
    ++launches;
    for (uint32_t chosen = 1; chosen < k; ++chosen) {
      const double total = seq_sum(nearest.p, true);
      uint64_t picked;
      if (total <= 0.0) {
        picked = rng.gen_index(n);
      } else {
        const double target = rng.gen_f64(0.0, total);
        launches += summer.enqueue_search(nearest.p, n, target, s);
        PXC_CUDA(cudaMemcpyAsync(h_u64, summer.found.p, sizeof(unsigned long long), cudaMemcpyDeviceToHost, s));
        PXC_CUDA(cudaStreamSynchronize(s));
        picked = h_u64[0];
      }
      float* c = cur.p + (size_t)chosen * ldc;
      PXC_CUDA(cudaMemcpyAsync(c, P + picked * ldp, d * sizeof(float), cudaMemcpyDeviceToDevice, s));
      kpp_update_kernel<<<blocks(n, pb), pb, exact_smem(pb), s>>>(P, ldp, n, d, c, nearest.p, 0);
      ++launches;
      PXC_CUDA(cudaGetLastError());
    }
  }

  Result run(uint32_t max_iter, const float* d_init, ChaCha8* rng) {
    Result r;
    r.k = k;
    r.path = tensor ? 1 : 0;
    if (d_init)
      PXC_CUDA(cudaMemcpy2DAsync(cur.p, ldc * 4, d_init, d * 4, d * 4, k, cudaMemcpyDeviceToDevice, s));
    else
      seed_kpp(*rng);
    const int sort_bits = std::max(1, 32 - __builtin_clz(std::max<uint32_t>(k - 1, 1)));
    for (uint32_t it = 0; it < max_iter; ++it) {
      r.iterations = it + 1;
      mark(2);
      nearest_pass(cur.p, it > 0, &r.rescanned);
      mark(3);
      PXC_CUDA(cudaMemcpyAsync(h_words + 4, words.p, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
      r.inertia = seq_sum(bestd.p, false);  // synchronises
      bool changed = h_words[4] != 0;
      if (sharded) exchange_progress(r.inertia, changed);
      if (!changed && it > 0) break;
      if (sharded) {
        sharded_update(sort_bits);
        mark(4);
        if (read_word(2)) reseed_empty(r);
        mark(5);
        std::swap(cur.p, next.p);
        continue;
      }
      // update: stable sort by cluster, per-cluster sums in point order
      size_t tb = sort_tmp_bytes;
      PXC_CUDA(cub::DeviceRadixSort::SortPairs(sort_tmp.p, tb, assign.p, keys_b.p, iota.p, sorted.p, (int)n, 0,
                                               sort_bits, s));
      offsets_kernel<<<blocks(k + 1, 256), 256, 0, s>>>(keys_b.p, n, k, off.p);
      PXC_CUDA(cudaMemsetAsync(words.p + 2, 0, sizeof(uint32_t), s));
      const uint32_t groups = (d + 31) / 32;
      cluster_mean_kernel<<<blocks((uint64_t)k * groups * 32, 256), 256, 0, s>>>(P, ldp, d, groups, sorted.p, off.p, k,
                                                                               next.p, ldc, words.p + 2);
      launches += 3;
      PXC_CUDA(cudaGetLastError());
      mark(4);
      const uint32_t empties = read_word(2);
      if (empties) reseed_empty(r);
      mark(5);
      if (trace)
        std::fprintf(stderr, "[pxc kmeans] iteration %u: assign %.3f ms, inertia+update %.3f ms, %u re-seeds %.3f ms\n",
                     it, span(2, 3), span(3, 4), empties, span(4, 5));
      std::swap(cur.p, next.p);
    }
    return r;
  }

  // Sharded: the ranks' inertia (f64 partial sums, added in rank order) and
  // `changed` flags (any) of the assignment pass.
  void exchange_progress(double& inertia, bool& changed) {
    struct alignas(16) Progress {
      double inertia;
      uint32_t changed, pad;
    };
    const int nr = ctx->nranks;
    xs.reserve(sizeof(Progress));
    xr.reserve(sizeof(Progress) * nr);
    Progress mine{inertia, changed ? 1u : 0u, 0u};
    PXC_CUDA(cudaMemcpyAsync(xs.p, &mine, sizeof(mine), cudaMemcpyHostToDevice, s));
    comm_allgather(ctx, xs.p, xr.p, sizeof(Progress), s, "k-means progress exchange");
    std::vector<Progress> all(nr);
    PXC_CUDA(cudaMemcpy(all.data(), xr.p, sizeof(Progress) * nr, cudaMemcpyDeviceToHost));
    double total = 0.0;
    bool any = false;
    for (const Progress& p : all) {
      total += p.inertia;
      any |= p.changed != 0;
    }
    inertia = total;
    changed = any;
  }

  // Sharded update: local per-cluster sums and counts, one allgather, the
  // rank-ordered fold into next; words[2] counts the globally empty clusters.
  void sharded_update(int sort_bits) {
    size_t tb = sort_tmp_bytes;
    PXC_CUDA(cub::DeviceRadixSort::SortPairs(sort_tmp.p, tb, assign.p, keys_b.p, iota.p, sorted.p, (int)n, 0,
                                             sort_bits, s));
    offsets_kernel<<<blocks(k + 1, 256), 256, 0, s>>>(keys_b.p, n, k, off.p);
    const size_t seg = ((size_t)k * d * 8 + (size_t)k * 4 + 15) / 16 * 16;
    xs.reserve(seg);
    xr.reserve(seg * ctx->nranks);
    const uint32_t groups = (d + 31) / 32;
    cluster_sum_kernel<<<blocks((uint64_t)k * groups * 32, 256), 256, 0, s>>>(
        P, ldp, d, groups, sorted.p, off.p, k, reinterpret_cast<double*>(xs.p),
        reinterpret_cast<uint32_t*>(xs.p + (size_t)k * d * 8));
    PXC_CUDA(cudaGetLastError());
    launches += 3;
    comm_allgather(ctx, xs.p, xr.p, seg, s, "k-means update exchange");
    gcount.reserve(k);
    PXC_CUDA(cudaMemsetAsync(words.p + 2, 0, sizeof(uint32_t), s));
    fold_means_kernel<<<blocks((uint64_t)k * d, 256), 256, 0, s>>>(xr.p, seg, ctx->nranks, k, d, next.p, ldc,
                                                                   gcount.p, words.p + 2);
    PXC_CUDA(cudaGetLastError());
    launches += 1;
  }

  // Sharded re-seeding of cluster e: the ranks' farthest points exchanged,
  // the global one copied into next[e] on every rank.
  void sharded_farthest(uint32_t e, const unsigned long long* local_key) {
    const size_t seg = (16 + (size_t)d * 4 + 15) / 16 * 16;
    xs.reserve(seg);
    xr.reserve(seg * ctx->nranks);
    farthest_candidate_kernel<<<1, 128, 0, s>>>(P, ldp, d, local_key, global_first, xs.p);
    comm_allgather(ctx, xs.p, xr.p, seg, s, "k-means re-seed exchange");
    farthest_pick_kernel<<<1, 128, 0, s>>>(xr.p, seg, ctx->nranks, d, next.p + (size_t)e * ldc);
    PXC_CUDA(cudaGetLastError());
    launches += 2;
  }

  // Empty clusters, in index order (kmeans.rs:118-126): each takes the
  // farthest point (kmeans.rs:215-226) against the centroids as they stand
  // at that moment — [0, e) already updated (in next, earlier re-seeds
  // included) and [e, k) not yet (cur).
  //
  // Exact and pruned with the bounds above: the points with the largest
  // bounds are scanned exactly first; only points whose bound reaches the
  // best of those can still be the farthest, and they are scanned exactly
  // too. Scanned points keep their exact distance as a tight bound for the
  // following empty clusters.
  void reseed_empty(Result& r) {
    std::vector<uint32_t> offs(k + 1);
    PXC_CUDA(cudaMemcpyAsync(offs.data(), off.p, (k + 1) * sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    if (sharded) {  // emptiness is global: the folded counts
      h_gcount.resize(k);
      PXC_CUDA(cudaMemcpyAsync(h_gcount.data(), gcount.p, k * sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    }
    pair_l2_kernel<false><<<blocks(n, 128), 128, 0, s>>>(P, ldp, n, d, next.p, ldc, assign.p, u_next.p);
    // bounds: the exact distance to the old centroid of the point's cluster
    PXC_CUDA(cudaMemcpyAsync(ub.p, bestd.p, n * 4, cudaMemcpyDeviceToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(ubc.p, assign.p, n * 4, cudaMemcpyDeviceToDevice, s));
    PXC_CUDA(cudaMemsetAsync(ube.p, 0, n * 4, s));
    launches += 1;
    PXC_CUDA(cudaStreamSynchronize(s));
    const uint32_t cap = (uint32_t)std::min<uint64_t>(8 * SEEDS, n);
    for (uint32_t e = 0; e < k; ++e) {
      if (sharded ? h_gcount[e] != 0 : offs[e] != offs[e + 1]) continue;
      if (e) PXC_CUDA(cudaMemcpyAsync(part.p, next.p, (size_t)e * ldc * 4, cudaMemcpyDeviceToDevice, s));
      PXC_CUDA(cudaMemcpyAsync(part.p + (size_t)e * ldc, cur.p + (size_t)e * ldc, (size_t)(k - e) * ldc * 4,
                               cudaMemcpyDeviceToDevice, s));
      // seeds: exact distances for the best-bounded points; the best in key[0];
      // then every point whose bound reaches it
      auto seed_and_filter = [&]() -> uint32_t {
        PXC_CUDA(cudaMemsetAsync(key.p, 0, 2 * sizeof(unsigned long long), s));
        PXC_CUDA(cudaMemsetAsync(words.p + 1, 0, 3 * sizeof(uint32_t), s));
        PXC_CUDA(cudaMemsetAsync(hist.p, 0, 4096 * sizeof(uint32_t), s));
        ub_hist_kernel<<<ctx->sm_count * 2, 512, 0, s>>>(P, ldp, n, d, next.p, ldc, assign.p, u_next.p, bestd.p, e,
                                                          ub.p, ubc.p, ube.p, hist.p);
        ub_level1_kernel<<<1, 256, 0, s>>>(hist.p, SEEDS, hist.p + 4096);
        ub_hist2_kernel<<<ctx->sm_count * 2, 512, 0, s>>>(ub.p, n, hist.p, hist.p + 4096);
        ub_level2_kernel<<<1, 256, 0, s>>>(hist.p, SEEDS, hist.p + 4096);
        ub_gather_kernel<<<ctx->sm_count * 4, 256, 0, s>>>(ub.p, n, hist.p + 4096, cap, sorted.p, words.p + 3);
        clamp_count_kernel<<<1, 1, 0, s>>>(words.p + 3, cap);
        exact_list(part.p, sorted.p, words.p + 3, cap, ubc.p, ub.p, 2, ube.p, e);
        argmax_list_kernel<<<ctx->sm_count, 256, 0, s>>>(ub.p, sorted.p, words.p + 3, 0, key.p);
        ub_filter_kernel<<<ctx->sm_count * 4, 256, 0, s>>>(ub.p, n, key.p, rescan.p, words.p + 1);
        launches += 8;
        return read_word(1);
      };
      uint32_t nl = seed_and_filter();
      const uint32_t nl_cheap = nl;
      if (nl > SCREEN_FALLBACK && tensor) {
        // the cheap bounds are loose here: bound every point by a screening pass
        const uint64_t kpad = (uint64_t)ntiles * km_tc::BN;
        PXC_CUDA(cudaMemsetAsync(words.p + 4, 0, sizeof(uint32_t), s));
        sqnorm_kernel<<<blocks(kpad * 32, 256), 256, 0, s>>>(part.p, ldc, k, d, kpad, cnorm.p, words.p + 4);
        screen(part.p, true);
        ub_screened_kernel<<<blocks(n, 256), 256, 0, s>>>(n, d, pnorm.p, words.p + 4, amin.p, e, ub.p, ubc.p, ube.p);
        launches += 2;
        nl = seed_and_filter();
      }
      if (trace)
        std::fprintf(stderr, "[pxc kmeans] reseed cluster %u: %u points can be the farthest (%u before screening)\n",
                     e, nl, nl_cheap);
      exact_list(part.p, rescan.p, words.p + 1, nl, ubc.p, ub.p, 2, ube.p, e);
      argmax_list_kernel<<<ctx->sm_count * 4, 256, 0, s>>>(ub.p, rescan.p, words.p + 1, 0, key.p + 1);
      if (sharded)
        sharded_farthest(e, key.p + 1);
      else
        copy_row_kernel<<<1, 128, 0, s>>>(P, ldp, d, key.p + 1, next.p + (size_t)e * ldc);
      launches += 2;
      PXC_CUDA(cudaGetLastError());
      ++r.reseeded;
    }
  }
};

// `d_pts` has a pitch of `ld` floats. The tensor path needs a 16-byte aligned
// base and a pitch that is a multiple of 4 floats; other layouts are copied.
// Prepares a Runner over d_pts (pitch ld): validation, layout, workspace.
// Returns false when there is nothing to cluster (n or d zero).
static void prepare_runner(Runner& R, pxc_ctx* ctx, const float* d_pts, uint32_t ld, uint64_t n, uint32_t d,
                           uint32_t k_eff, DBuf<float>& padded, cudaStream_t s, bool allow_tensor);

Result kmeans_impl(pxc_ctx* ctx, const float* d_pts, uint32_t ld, uint64_t n, uint32_t d, uint32_t k,
                   uint32_t max_iter, const float* d_init, ChaCha8* rng, float* d_out_cent, uint32_t* d_out_assign,
                   cudaStream_t s) {
  Result r;
  const uint64_t n_eff = d == 0 ? 0 : n;
  const uint32_t k_eff = (uint32_t)std::max<uint64_t>(std::min<uint64_t>(k, n_eff), 1);
  r.k = k_eff;
  if (n_eff == 0) {
    if (d) PXC_CUDA(cudaMemsetAsync(d_out_cent, 0, (size_t)k_eff * d * 4, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    return r;
  }
  PXC_CONFIG(d <= MAX_DIM, "dim", d, "k-means on the device supports dim <= 512");
  PXC_CONFIG(n <= 0x7FFFFFFFull, "n", n, "k-means on the device supports fewer than 2^31 points");
  Runner R(workspace(ctx));
  DBuf<float> padded;
  prepare_runner(R, ctx, d_pts, ld, n, d, k_eff, padded, s, true);
  r = R.run(max_iter, d_init, rng);
  r.k = k_eff;
  r.screen_passes = R.screen_passes;
  r.screen_ms = R.screen_ms;
  PXC_CUDA(cudaMemcpy2DAsync(d_out_cent, d * 4, R.cur.p, R.ldc * 4, d * 4, k_eff, cudaMemcpyDeviceToDevice, s));
  if (d_out_assign) PXC_CUDA(cudaMemcpyAsync(d_out_assign, R.assign.p, n * 4, cudaMemcpyDeviceToDevice, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  check_device_status(ctx, s, "k-means");
  ctx->launches += R.launches;
  return r;
}

// proxima_quantize::kmeans over points sharded across the ranks of the
// context's communicator, from an injected init (identical on every rank).
// Assignments are exact per point; the per-cluster f64 sums are folded in
// rank order, so centroids equal a single run's whenever those sums are
// exact, and are within rounding of it otherwise.
Result kmeans_sharded_impl(pxc_ctx* ctx, const float* d_pts, uint32_t ld, uint64_t n, uint32_t d, uint32_t k,
                           uint32_t max_iter, const float* d_init, float* d_out_cent, uint32_t* d_out_assign,
                           cudaStream_t s) {
  PXC_CONFIG(d >= 1 && d <= MAX_DIM, "dim", d, "k-means on the device supports 1 <= dim <= 512");
  PXC_CONFIG(n >= 1 && n <= 0x7FFFFFFFull, "n", n, "every rank holds between 1 and 2^31 - 1 points");
  PXC_CONFIG(d_init != nullptr, "init", 0, "the sharded k-means starts from an injected init");
  std::lock_guard<std::mutex> comm_lock(ctx->comm_mu);
  // the global point order: ranks hold consecutive ranges
  const int nr = ctx->nranks;
  DBuf<uint64_t> cnt_s, cnt_r;
  cnt_s.reserve(2);
  cnt_r.reserve(2 * (size_t)nr);
  const uint64_t mine[2] = {n, 0};
  PXC_CUDA(cudaMemcpyAsync(cnt_s.p, mine, sizeof(mine), cudaMemcpyHostToDevice, s));
  comm_allgather(ctx, cnt_s.p, cnt_r.p, sizeof(mine), s, "k-means point counts");
  std::vector<uint64_t> counts(2 * (size_t)nr);
  PXC_CUDA(cudaMemcpy(counts.data(), cnt_r.p, counts.size() * 8, cudaMemcpyDeviceToHost));
  uint64_t n_global = 0, first = 0;
  for (int r = 0; r < nr; ++r) {
    if (r == ctx->rank) first = n_global;
    n_global += counts[2 * r];
  }
  const uint32_t k_eff = (uint32_t)std::max<uint64_t>(std::min<uint64_t>(k, n_global), 1);
  Runner R(workspace(ctx));
  DBuf<float> padded;
  prepare_runner(R, ctx, d_pts, ld, n, d, k_eff, padded, s, true);
  R.sharded = true;
  R.global_first = first;
  Result r = R.run(max_iter, d_init, nullptr);
  r.k = k_eff;
  r.screen_passes = R.screen_passes;
  r.screen_ms = R.screen_ms;
  PXC_CUDA(cudaMemcpy2DAsync(d_out_cent, d * 4, R.cur.p, R.ldc * 4, d * 4, k_eff, cudaMemcpyDeviceToDevice, s));
  if (d_out_assign) PXC_CUDA(cudaMemcpyAsync(d_out_assign, R.assign.p, n * 4, cudaMemcpyDeviceToDevice, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  check_device_status(ctx, s, "k-means");
  ctx->launches += R.launches;
  return r;
}

static void prepare_runner(Runner& R, pxc_ctx* ctx, const float* d_pts, uint32_t ld, uint64_t n, uint32_t d,
                           uint32_t k_eff, DBuf<float>& padded, cudaStream_t s, bool allow_tensor) {
  R.ctx = ctx;
  R.s = s;
  R.n = n;
  R.d = d;
  R.k = k_eff;
  R.ldc = (d + 3) & ~3u;
  if ((reinterpret_cast<uintptr_t>(d_pts) & 15) == 0 && (ld & 3) == 0) {
    R.P = d_pts;
    R.ldp = ld;
  } else {
    R.ldp = (d + 3) & ~3u;
    padded.reserve((size_t)n * R.ldp);
    PXC_CUDA(cudaMemsetAsync(padded.p, 0, (size_t)n * R.ldp * 4, s));
    PXC_CUDA(cudaMemcpy2DAsync(padded.p, R.ldp * 4, d_pts, (size_t)ld * 4, d * 4, n, cudaMemcpyDeviceToDevice, s));
    R.P = padded.p;
  }
  // validation: finite, and magnitudes for which the screening bounds hold
  DBuf<unsigned long long> bad;
  bad.reserve(1);
  DBuf<uint32_t> mx;
  mx.reserve(1);
  PXC_CUDA(cudaMemsetAsync(bad.p, 0xFF, 8, s));
  PXC_CUDA(cudaMemsetAsync(mx.p, 0, 4, s));
  scan_input_kernel<<<ctx->sm_count * 8, 256, 0, s>>>(R.P, R.ldp, n, d, bad.p, mx.p);
  R.launches++;
  unsigned long long* hs = R.h_u64 + 1;
  hs[0] = hs[1] = 0;
  PXC_CUDA(cudaMemcpyAsync(hs, bad.p, 8, cudaMemcpyDeviceToHost, s));
  PXC_CUDA(cudaMemcpyAsync(hs + 1, mx.p, 4, cudaMemcpyDeviceToHost, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  const unsigned long long hb = hs[0];
  const uint32_t hm = (uint32_t)hs[1];
  if (hb != ~0ull) throw make_failure(PXC_NON_FINITE, hb, 0, "points", "point element %llu is not finite", hb);
  float maxabs;
  std::memcpy(&maxabs, &hm, 4);
  const bool want_tensor = !ctx->opt_kmeans_exact && d >= 16 && d <= 32u * km_tc::MAX_KBLOCKS &&
                           k_eff >= 256 && n >= 256 && maxabs <= 0x1p40f;
  R.trace = ctx->opt_kmeans_trace;

  R.setup(want_tensor && allow_tensor);
}

// The caller's ChaCha8Rng state (pxc_rng) as a generator, and back.
ChaCha8 rng_from_abi(const pxc_rng* r) {
  PXC_CONFIG(r->word_pos_hi < 16, "word_pos", r->word_pos_hi, "ChaCha8Rng word positions are below 2^68");
  return ChaCha8(r->seed, r->stream, r->word_pos_lo, r->word_pos_hi);
}
void rng_to_abi(const ChaCha8& g, pxc_rng* r) { g.state(r->seed, &r->stream, &r->word_pos_lo, &r->word_pos_hi); }

// kmeans drawing k-means++ from the caller's generator (advanced in place), or from an init.
Result kmeans_device(pxc_ctx* ctx, const float* d_pts, uint32_t ld, uint64_t n, uint32_t d, uint32_t k,
                     uint32_t max_iter, const float* d_init, pxc_rng* rng, float* d_out_cent,
                     uint32_t* d_out_assign, cudaStream_t s) {
  const bool draws = d_init == nullptr && n > 0 && d > 0;
  PXC_CONFIG(!draws || rng != nullptr, "rng", 0, "k-means++ seeding needs the caller's generator (rng is null)");
  if (!draws) return kmeans_impl(ctx, d_pts, ld, n, d, k, max_iter, d_init, nullptr, d_out_cent, d_out_assign, s);
  ChaCha8 g = rng_from_abi(rng);
  Result r = kmeans_impl(ctx, d_pts, ld, n, d, k, max_iter, d_init, &g, d_out_cent, d_out_assign, s);
  rng_to_abi(g, rng);
  return r;
}

// Exact nearest centroid of every row (ties to the lower index): `unrolled`
// selects squared_euclidean's 8-lane order (IvfPqIndex's nearest_centroid,
// ivfpq.rs:1231-1243), else the sequential one. Centroids: k x d, pitch d.
void nearest_rows(pxc_ctx* ctx, const float* d_pts, uint32_t ld, uint64_t n, uint32_t d, const float* d_cent,
                  uint32_t k, bool unrolled, uint32_t* d_assign, float* d_dist, cudaStream_t s) {
  if (n == 0) return;
  Runner R(workspace(ctx));
  DBuf<float> padded;
  R.unrolled = unrolled;
  prepare_runner(R, ctx, d_pts, ld, n, d, k, padded, s, true);
  PXC_CUDA(cudaMemcpy2DAsync(R.cur.p, R.ldc * 4, d_cent, d * 4, d * 4, k, cudaMemcpyDeviceToDevice, s));
  uint64_t rescanned = 0;
  R.nearest_pass(R.cur.p, false, &rescanned);
  PXC_CUDA(cudaMemcpyAsync(d_assign, R.assign.p, n * 4, cudaMemcpyDeviceToDevice, s));
  if (d_dist) PXC_CUDA(cudaMemcpyAsync(d_dist, R.bestd.p, n * 4, cudaMemcpyDeviceToDevice, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  check_device_status(ctx, s, "nearest centroid");
  ctx->launches += R.launches;
}

void fill_info(pxc_kmeans_info* info, const Result& r) {
  if (!info) return;
  std::memset(info, 0, sizeof(*info));
  info->k = r.k;
  info->iterations = r.iterations;
  info->inertia = r.inertia;
  info->path = r.path;
  info->reseeded = r.reseeded;
  info->rescanned = r.rescanned;
  info->screen_passes = r.screen_passes;
  info->screen_ms = r.screen_ms;
}

}  // namespace km
}  // namespace pxc

using namespace pxc;

extern "C" {

pxc_status pxc_kmeans_device(pxc_ctx* ctx, const float* points, uint64_t n, uint32_t dim, uint32_t k,
                             uint32_t max_iterations, const float* init, pxc_rng* rng, float* out_centroids,
                             uint32_t* out_assign, pxc_kmeans_info* info, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(out_centroids != nullptr, "out_centroids", 0, "null output buffer");
    PXC_CONFIG(points != nullptr || n == 0 || dim == 0, "points", 0, "null point buffer");
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    km::Result r = km::kmeans_device(ctx, points, dim, n, dim, k, max_iterations, init, rng, out_centroids,
                                     out_assign, s);
    km::fill_info(info, r);
  });
}

pxc_status pxc_kmeans(pxc_ctx* ctx, const float* points, uint64_t n, uint32_t dim, uint32_t k,
                      uint32_t max_iterations, const float* init, pxc_rng* rng, float* out_centroids,
                      uint32_t* out_assign, pxc_kmeans_info* info, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(out_centroids != nullptr, "out_centroids", 0, "null output buffer");
    PXC_CONFIG(points != nullptr || n == 0 || dim == 0, "points", 0, "null point buffer");
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = ctx->stream;
    const uint64_t n_eff = dim == 0 ? 0 : n;
    const uint32_t k_eff = (uint32_t)std::max<uint64_t>(std::min<uint64_t>(k, n_eff), 1);
    const uint32_t ld = (dim + 3) & ~3u;
    DBuf<float> dp, dinit, dcent;
    DBuf<uint32_t> dassign;
    dp.reserve(std::max<size_t>(1, (size_t)n_eff * ld));
    dcent.reserve(std::max<size_t>(1, (size_t)k_eff * std::max<uint32_t>(dim, 1)));
    if (n_eff) {
      if (ld != dim) PXC_CUDA(cudaMemsetAsync(dp.p, 0, (size_t)n_eff * ld * 4, s));
      PXC_CUDA(cudaMemcpy2DAsync(dp.p, (size_t)ld * 4, points, (size_t)dim * 4, (size_t)dim * 4, n_eff,
                                 cudaMemcpyHostToDevice, s));
    }
    if (init && n_eff) {
      dinit.reserve((size_t)k_eff * dim);
      PXC_CUDA(cudaMemcpyAsync(dinit.p, init, (size_t)k_eff * dim * 4, cudaMemcpyHostToDevice, s));
    }
    if (out_assign && n_eff) dassign.reserve(n_eff);
    km::Result r = km::kmeans_device(ctx, dp.p, ld, n_eff, dim, k, max_iterations, init ? dinit.p : nullptr, rng,
                                     dcent.p, out_assign ? dassign.p : nullptr, s);
    if (dim) PXC_CUDA(cudaMemcpyAsync(out_centroids, dcent.p, (size_t)r.k * dim * 4, cudaMemcpyDeviceToHost, s));
    if (out_assign && n_eff)
      PXC_CUDA(cudaMemcpyAsync(out_assign, dassign.p, n_eff * 4, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    km::fill_info(info, r);
  });
}

pxc_status pxc_kmeans_sharded(pxc_ctx* ctx, const float* d_points, uint64_t n, uint32_t dim, uint32_t k,
                              uint32_t max_iterations, const float* d_init, float* d_out_centroids,
                              uint32_t* d_out_assign, pxc_kmeans_info* info, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(d_out_centroids != nullptr && d_points != nullptr, "points", 0, "null buffer");
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    km::Result r = km::kmeans_sharded_impl(ctx, d_points, dim, n, dim, k, max_iterations, d_init, d_out_centroids,
                                           d_out_assign, s);
    km::fill_info(info, r);
  });
}

pxc_status pxc_rng_seed_from_u64(uint64_t state, pxc_rng* out, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(out != nullptr, "out", 0, "null generator");
    km::rng_to_abi(ChaCha8(state), out);
  });
}

pxc_status pxc_rng_next_u32(pxc_rng* rng, uint32_t* out, uint64_t n, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(rng != nullptr, "rng", 0, "null generator");
    PXC_CONFIG(out != nullptr || n == 0, "out", 0, "null output buffer");
    ChaCha8 g = km::rng_from_abi(rng);
    for (uint64_t i = 0; i < n; ++i) out[i] = g.next_u32();
    km::rng_to_abi(g, rng);
  });
}

pxc_status pxc_rng_gen_index(pxc_rng* rng, uint64_t bound, uint64_t* out, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(rng != nullptr && out != nullptr, "rng", 0, "null generator or output");
    PXC_CONFIG(bound >= 1, "bound", bound, "gen_range(0..bound) needs bound >= 1");
    ChaCha8 g = km::rng_from_abi(rng);
    *out = g.gen_index(bound);
    km::rng_to_abi(g, rng);
  });
}

pxc_status pxc_rng_gen_f64(pxc_rng* rng, double low, double high, double* out, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(rng != nullptr && out != nullptr, "rng", 0, "null generator or output");
    PXC_CONFIG(low < high && std::isfinite(high - low), "high", 0, "gen_range(low..high) needs low < high, finite span");
    ChaCha8 g = km::rng_from_abi(rng);
    *out = g.gen_f64(low, high);
    km::rng_to_abi(g, rng);
  });
}

pxc_status pxc_chacha_block(const uint32_t key[8], uint64_t counter, uint64_t stream, uint32_t rounds,
                            uint32_t out[16], pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(key != nullptr && out != nullptr, "key", 0, "null key or output");
    PXC_CONFIG(rounds >= 2 && rounds <= 64 && rounds % 2 == 0, "rounds", rounds, "must be even, 2..64");
    chacha_block(key, counter, stream, (int)rounds, out);
  });
}

}  // extern "C"
