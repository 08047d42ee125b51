// refdist.cuh — distances in the reference's exact operation order.
//
// squared_euclidean_unrolled / dot_unrolled (crates/proxima-core/src/distance.rs:267-283,
// 317-331, reduce :534-538): lane i accumulates elements i, i+8, ...; the
// lanes are combined as ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)), then the tail
// (the remainder summed from 0.0) is added. Every step rounds separately
// (_rn intrinsics), so nvcc cannot contract them into FMAs.
#pragma once
#include <stdint.h>

namespace pxc {

__device__ __forceinline__ float l2_unrolled(const float* a, const float* __restrict__ b, uint32_t dim) {
  float acc[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) acc[l] = 0.0f;
  const uint32_t full = dim & ~7u;
  for (uint32_t i = 0; i < full; i += 8) {
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      const float d = __fsub_rn(a[i + l], __ldg(b + i + l));
      acc[l] = __fadd_rn(acc[l], __fmul_rn(d, d));
    }
  }
  float tail = 0.0f;
  for (uint32_t i = full; i < dim; ++i) {
    const float d = __fsub_rn(a[i], __ldg(b + i));
    tail = __fadd_rn(tail, __fmul_rn(d, d));
  }
  const float x = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
  const float y = __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7]));
  return __fadd_rn(__fadd_rn(x, y), tail);
}
__device__ __forceinline__ float dot_unrolled(const float* a, const float* __restrict__ b, uint32_t dim) {
  float acc[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) acc[l] = 0.0f;
  const uint32_t full = dim & ~7u;
  for (uint32_t i = 0; i < full; i += 8) {
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[l] = __fadd_rn(acc[l], __fmul_rn(a[i + l], __ldg(b + i + l)));
  }
  float tail = 0.0f;
  for (uint32_t i = full; i < dim; ++i) tail = __fadd_rn(tail, __fmul_rn(a[i], __ldg(b + i)));
  const float x = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
  const float y = __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7]));
  return __fadd_rn(__fadd_rn(x, y), tail);
}
// space.distance for the metrics IVF-PQ reranks with (space.rs:148-156).

}  // namespace pxc
