// topk.cuh — block-level sorting helpers shared by the merge kernels.
//
// TopK in the reference (crates/proxima-core/src/topk.rs:93-191) keeps the k
// smallest SearchResults under (f32::total_cmp(distance), id). Every device
// selection here produces exactly that set, then sorts it in that order.
#pragma once
#include <stdint.h>

namespace pxc {

// In-place ascending bitonic sort of n (power of two) u64 keys in shared
// memory by the whole block.
__device__ inline void block_bitonic_sort_u64(uint64_t* s, uint32_t n) {
  for (uint32_t size = 2; size <= n; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (uint32_t i = threadIdx.x; i < (n >> 1); i += blockDim.x) {
        uint32_t lo = 2 * i - (i & (stride - 1));
        uint32_t hi = lo + stride;
        bool up = ((lo & size) == 0);
        uint64_t a = s[lo], b = s[hi];
        if ((a > b) == up) {
          s[lo] = b;
          s[hi] = a;
        }
      }
    }
  }
  __syncthreads();
}

// Same, for (order key, id) pairs compared lexicographically.
__device__ inline void block_bitonic_sort_key_id(uint32_t* key, uint64_t* id, uint32_t n) {
  for (uint32_t size = 2; size <= n; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (uint32_t i = threadIdx.x; i < (n >> 1); i += blockDim.x) {
        uint32_t lo = 2 * i - (i & (stride - 1));
        uint32_t hi = lo + stride;
        bool up = ((lo & size) == 0);
        uint32_t ka = key[lo], kb = key[hi];
        uint64_t ia = id[lo], ib = id[hi];
        bool greater = (ka > kb) || (ka == kb && ia > ib);
        if (greater == up) {
          key[lo] = kb;
          key[hi] = ka;
          id[lo] = ib;
          id[hi] = ia;
        }
      }
    }
  }
  __syncthreads();
}

}  // namespace pxc
