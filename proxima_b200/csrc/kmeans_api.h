// kmeans_api.h — the k-means machinery (kmeans.cu) as used by the IVF-PQ
// build (ivfpq.cu): clustering with a caller-owned ChaCha8 stream, and exact
// nearest-centroid assignment in either summation order.
#pragma once
#include <stdint.h>

#include "common.cuh"
#include "rng.h"

namespace pxc {
namespace km {

struct Result {
  uint32_t k = 0, iterations = 0, path = 0, reseeded = 0;
  uint64_t rescanned = 0;
  double inertia = 0.0;
  uint32_t screen_passes = 0;
  float screen_ms = 0.0f;
};

// proxima_quantize::kmeans on device rows (pitch ld floats): k-means++ from
// `rng` (advanced in place, as the reference's &mut ChaCha8Rng) unless d_init
// is given. d_out_cent: k_eff x d, pitch d.
Result kmeans_impl(pxc_ctx* ctx, const float* d_pts, uint32_t ld, uint64_t n, uint32_t d, uint32_t k,
                   uint32_t max_iter, const float* d_init, ChaCha8* rng, float* d_out_cent, uint32_t* d_out_assign,
                   cudaStream_t s);

// Exact nearest centroid of every row, ties to the lower index; `unrolled`
// selects proxima_core::distance::squared_euclidean's 8-lane order, else the
// sequential order of kmeans.rs `squared`. Centroids k x d, pitch d.
void nearest_rows(pxc_ctx* ctx, const float* d_pts, uint32_t ld, uint64_t n, uint32_t d, const float* d_cent,
                  uint32_t k, bool unrolled, uint32_t* d_assign, float* d_dist, cudaStream_t s);

}  // namespace km
}  // namespace pxc
