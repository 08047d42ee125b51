// hostcopy.cuh — copies between PAGEABLE host memory and the device at the
// copy engine's rate. A copy from pageable memory through the driver is staged
// one chunk at a time by one thread; here host threads fill (or drain) a ring
// of pinned chunks while the copy engine moves the previous chunk, so the
// host's memory bandwidth and the link run concurrently. Pinned or registered
// host memory goes straight to cudaMemcpyAsync.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace pxc {
namespace hostcopy {

// dst (device) <- src (host), ordered on `s`. Returns once every byte of
// `src` has been read (the ring's last copies may still be in flight on `s`).
void to_device(pxc_ctx* ctx, void* dst, const void* src, size_t n, cudaStream_t s);
// dst (host) <- src (device): the stream's earlier work comes first; returns
// once every byte is in `dst`.
void to_host(pxc_ctx* ctx, void* dst, const void* src, size_t n, cudaStream_t s);
// Frees the context's ring and threads (called by pxc_ctx_destroy).
void release(void* stager);

}  // namespace hostcopy
}  // namespace pxc
