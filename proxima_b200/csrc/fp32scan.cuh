// fp32scan.cuh — reference-order fp32 distances on CUDA cores: the per-lane
// step and lane reduction of crates/proxima-core/src/distance.rs, and the
// tiled distance kernel used by the generic flat scan and the IVF coarse
// search. Every float operation is an _rn intrinsic so nvcc cannot contract
// it into an FMA.
#pragma once
#include <stdint.h>

#include "common.cuh"
#include "select.cuh"

namespace pxc {

// ---------------------------------------------------------------------------
// Reference-order distance (crates/proxima-core/src/distance.rs). All float
// operations use the _rn intrinsics so nvcc cannot contract them into FMAs.
// ---------------------------------------------------------------------------
template <int METRIC>
__device__ __forceinline__ float lane_step(float acc, float q, float x) {
  if (METRIC == PXC_EUCLIDEAN) {
    float d = __fsub_rn(q, x);
    return __fadd_rn(acc, __fmul_rn(d, d));
  } else if (METRIC == PXC_MANHATTAN) {
    return __fadd_rn(acc, fabsf(__fsub_rn(q, x)));
  } else {
    return __fadd_rn(acc, __fmul_rn(q, x));
  }
}

template <int METRIC>
__device__ __forceinline__ float finish(const float (&acc)[8], float tail) {
  float a = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
  float b = __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7]));
  float s = __fadd_rn(__fadd_rn(a, b), tail);
  if (METRIC == PXC_COSINE) return __fsub_rn(1.0f, s);
  if (METRIC == PXC_INNER_PRODUCT) return -s;
  return s;
}

__device__ inline bool accepted(const uint64_t* bitmap, uint32_t slot) {
  return bitmap == nullptr || ((bitmap[slot >> 6] >> (slot & 63)) & 1ull);
}

__device__ inline uint32_t candidate_key(float d) {
  uint32_t k = order_key(d);
  return k == SENTINEL ? SENTINEL - 1 : k;  // keep the sentinel unambiguous
}

// K1g: distance tile of 32 queries x 64 rank rows, written as order keys into
// D[q][r - c0] (row stride C). With a bitmap, row r is kept when the bitmap
// accepts slot rank_slot[r] (rank_slot may be null without a bitmap). Thread (tq, tr) owns queries {tq, tq+16} and
// rows {tr, tr+16, tr+32, tr+48}, each pair with eight lane accumulators.
template <int METRIC>
__global__ void __launch_bounds__(256) dist_chunk_kernel(
    const float* __restrict__ Q, uint32_t nq, const float* __restrict__ X, uint64_t nrank,
    uint32_t dim, uint64_t c0, uint32_t C, const uint64_t* __restrict__ bitmap,
    const uint32_t* __restrict__ rank_slot, uint32_t* __restrict__ D) {
  __shared__ __align__(16) float sQ[32][36];
  __shared__ __align__(16) float sX[64][36];
  const int t = threadIdx.x, tq = t >> 4, tr = t & 15;
  const uint32_t q0 = blockIdx.y * 32;
  const uint64_t r0 = c0 + (uint64_t)blockIdx.x * 64;
  float acc[2][4][8];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int l = 0; l < 8; ++l) acc[a][b][l] = 0.0f;
  const uint32_t full = dim / 8 * 8;
  for (uint32_t k0 = 0; k0 < full; k0 += 32) {
    const uint32_t kw = min(32u, full - k0);
    for (int i = t; i < 32 * 32; i += 256) {
      int row = i >> 5, col = i & 31;
      uint32_t q = q0 + row;
      sQ[row][col] = (q < nq && (uint32_t)col < kw) ? Q[(size_t)q * dim + k0 + col] : 0.0f;
    }
    for (int i = t; i < 64 * 32; i += 256) {
      int row = i >> 5, col = i & 31;
      uint64_t r = r0 + row;
      sX[row][col] = (r < nrank && (uint32_t)col < kw) ? X[r * dim + k0 + col] : 0.0f;
    }
    __syncthreads();
    for (uint32_t g = 0; g < kw; g += 8) {
      float qv[2][8], xv[4][8];
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        float4 u = *reinterpret_cast<const float4*>(&sQ[tq + 16 * a][g]);
        float4 w = *reinterpret_cast<const float4*>(&sQ[tq + 16 * a][g + 4]);
        qv[a][0] = u.x; qv[a][1] = u.y; qv[a][2] = u.z; qv[a][3] = u.w;
        qv[a][4] = w.x; qv[a][5] = w.y; qv[a][6] = w.z; qv[a][7] = w.w;
      }
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        float4 u = *reinterpret_cast<const float4*>(&sX[tr + 16 * b][g]);
        float4 w = *reinterpret_cast<const float4*>(&sX[tr + 16 * b][g + 4]);
        xv[b][0] = u.x; xv[b][1] = u.y; xv[b][2] = u.z; xv[b][3] = u.w;
        xv[b][4] = w.x; xv[b][5] = w.y; xv[b][6] = w.z; xv[b][7] = w.w;
      }
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
          for (int l = 0; l < 8; ++l) acc[a][b][l] = lane_step<METRIC>(acc[a][b][l], qv[a][l], xv[b][l]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    const uint32_t q = q0 + tq + 16 * a;
    if (q >= nq) continue;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint64_t r = r0 + tr + 16 * b;
      uint32_t key = SENTINEL;
      if (r < nrank && (bitmap == nullptr || accepted(bitmap, rank_slot[r]))) {
        float tail = 0.0f;  // the remainder loop starts from 0.0 (distance.rs:277-281)
        for (uint32_t d = full; d < dim; ++d)
          tail = lane_step<METRIC>(tail, Q[(size_t)q * dim + d], X[r * dim + d]);
        key = candidate_key(finish<METRIC>(acc[a][b], tail));
      }
      D[(size_t)q * C + (r - c0)] = key;
    }
  }
}

}  // namespace pxc
