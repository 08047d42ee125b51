// ctx.cu — device context and the multi-GPU candidate merge.
#include <algorithm>
#include <new>

#include "common.cuh"
#include "topk.cuh"

namespace pxc {

void check_device_status(pxc_ctx* ctx, cudaStream_t s, const char* where) {
  check_status_word(ctx->d_status, ctx->h_status, s, where);
}

void check_status_word(uint32_t* d_status, uint32_t* h_status, cudaStream_t s, const char* where) {
  PXC_CUDA(cudaMemcpyAsync(h_status, d_status, 2 * sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  uint32_t code = h_status[0];
  if (code != DEV_OK) {
    uint32_t aux = h_status[1];
    PXC_CUDA(cudaMemsetAsync(d_status, 0, 2 * sizeof(uint32_t), s));
    PXC_CUDA(cudaStreamSynchronize(s));
    if (code == DEV_BAD_SHAPE)
      throw make_failure(PXC_INTERNAL, code, aux, nullptr, "%s: kernel rejected its launch shape",
                         where);
    throw make_failure(PXC_TIMEOUT, code, aux, nullptr,
                       "%s: a bounded device wait gave up (code %u, block %u)", where, code, aux);
  }
}

// One warp-free block per query: gather the union of the parts, sort by
// (total_cmp(distance), id), keep k.
__global__ void merge_parts_kernel(const uint64_t* __restrict__ ids, const float* __restrict__ dist,
                                   const uint32_t* __restrict__ lens, uint32_t nparts, uint32_t nq,
                                   uint32_t k_in, uint32_t k, uint32_t cap,
                                   uint64_t* __restrict__ out_ids, float* __restrict__ out_dist,
                                   uint32_t* __restrict__ out_len) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint32_t* skey = reinterpret_cast<uint32_t*>(smem_raw);
  uint64_t* sid = reinterpret_cast<uint64_t*>(smem_raw + cap * sizeof(uint32_t) +
                                              ((cap * sizeof(uint32_t)) & 4));
  uint32_t q = blockIdx.x;
  if (q >= nq) return;
  __shared__ uint32_t count;
  if (threadIdx.x == 0) count = 0;
  __syncthreads();
  for (uint32_t p = 0; p < nparts; ++p) {
    uint32_t len = min(lens[(size_t)p * nq + q], k_in);
    for (uint32_t i = threadIdx.x; i < len; i += blockDim.x) {
      uint32_t pos = atomicAdd(&count, 1u);
      size_t src = ((size_t)p * nq + q) * k_in + i;
      skey[pos] = order_key(dist[src]);
      sid[pos] = ids[src];
    }
  }
  __syncthreads();
  uint32_t n = count;
  for (uint32_t i = n + threadIdx.x; i < cap; i += blockDim.x) {
    skey[i] = 0xFFFFFFFFu;
    sid[i] = ~0ull;
  }
  __syncthreads();
  block_bitonic_sort_key_id(skey, sid, cap);
  uint32_t take = min(n, k);
  for (uint32_t i = threadIdx.x; i < take; i += blockDim.x) {
    out_ids[(size_t)q * k + i] = sid[i];
    out_dist[(size_t)q * k + i] = key_to_float(skey[i]);
  }
  if (threadIdx.x == 0) out_len[q] = take;
}

}  // namespace pxc

using namespace pxc;

extern "C" {

uint32_t pxc_abi_version(void) { return (1u << 16) | 0u; }

pxc_status pxc_ctx_create(const int* devices, int n_devices, pxc_ctx** out, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(out != nullptr, "out", 0, "output handle pointer is null");
    PXC_CONFIG(n_devices == 1 || (devices == nullptr && n_devices <= 1), "n_devices", n_devices,
               "one device per context; run one process per GPU and merge with pxc_topk_merge");
    int dev = devices ? devices[0] : 0;
    int count = 0;
    PXC_CUDA(cudaGetDeviceCount(&count));
    PXC_CONFIG(dev >= 0 && dev < count, "device", dev, "no such CUDA device");
    cudaDeviceProp prop;
    PXC_CUDA(cudaGetDeviceProperties(&prop, dev));
    PXC_CONFIG(prop.major == 10, "device", dev,
               "libproxima_cuda is built for sm_100a (B200) only");
    DeviceGuard g(dev);
    pxc_ctx* c = new (std::nothrow) pxc_ctx();
    if (!c) throw make_failure(PXC_INTERNAL, 0, 0, nullptr, "out of host memory");
    c->device = dev;
    c->sm_count = prop.multiProcessorCount;
    try {
      PXC_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
      PXC_CUDA(cudaMalloc(&c->d_status, 2 * sizeof(uint32_t)));
      PXC_CUDA(cudaMemset(c->d_status, 0, 2 * sizeof(uint32_t)));
      PXC_CUDA(cudaMallocHost(&c->h_status, 2 * sizeof(uint32_t)));
    } catch (...) {
      pxc_ctx_destroy(c);
      throw;
    }
    *out = c;
  });
}

void pxc_ctx_destroy(pxc_ctx* ctx) {
  if (!ctx) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  if (ctx->kmeans_ws && ctx->kmeans_ws_free) ctx->kmeans_ws_free(ctx->kmeans_ws);
  if (ctx->d_status) cudaFree(ctx->d_status);
  if (ctx->h_status) cudaFreeHost(ctx->h_status);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  if (prev >= 0) cudaSetDevice(prev);
  delete ctx;
}

pxc_status pxc_ctx_set_wait_limit(pxc_ctx* ctx, uint32_t milliseconds, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(milliseconds >= 1 && milliseconds <= 60000, "milliseconds", milliseconds,
               "must be between 1 and 60000");
    ctx->wait_ms = milliseconds;
  });
}

uint64_t pxc_ctx_launch_count(const pxc_ctx* ctx) { return ctx ? ctx->launches : 0; }

pxc_status pxc_ctx_set_option(pxc_ctx* ctx, const char* name, int64_t value, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(name != nullptr, "name", 0, "null option name");
    std::lock_guard<std::mutex> lock(ctx->mu);
    if (std::strcmp(name, "sq_candidate_cap") == 0) {
      ctx->opt_sq_candidate_cap = value < 0 ? -1 : value;
    } else if (std::strcmp(name, "sq_spec_rank") == 0) {
      ctx->opt_sq_spec_rank = value < 1 ? -1 : value;
    } else if (std::strcmp(name, "kmeans_exact") == 0) {
      ctx->opt_kmeans_exact = value != 0;
    } else if (std::strcmp(name, "kmeans_trace") == 0) {
      ctx->opt_kmeans_trace = value != 0;
    } else {
      throw make_failure(PXC_CONFIGURATION, 0, 0, "name", "unknown diagnostic option '%.64s'", name);
    }
  });
}

pxc_status pxc_ctx_set_profiling(pxc_ctx* ctx, int32_t on, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    ctx->profiling = on != 0;
  });
}

pxc_status pxc_topk_merge(pxc_ctx* ctx, const uint64_t* d_ids, const float* d_dist,
                          const uint32_t* d_lens, uint32_t nparts, uint32_t nq, uint32_t k_in,
                          uint32_t k, uint64_t* d_out_ids, float* d_out_dist,
                          uint32_t* d_out_len, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(k <= PXC_MAX_K, "k", k, "exceeds the 16777216 result ceiling");
    PXC_CONFIG(nparts >= 1, "nparts", nparts, "must be at least 1");
    uint64_t total = (uint64_t)nparts * k_in;
    PXC_CONFIG(total <= 8192, "nparts*k_in", total,
               "merge holds at most 8192 candidates per query");
    if (nq == 0) return;
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    uint32_t cap = 1;
    while (cap < total) cap <<= 1;
    if (cap < 32) cap = 32;
    size_t smem = cap * sizeof(uint32_t) + ((cap * sizeof(uint32_t)) & 4) + cap * sizeof(uint64_t);
    if (smem > 48 * 1024)
      PXC_CUDA(cudaFuncSetAttribute(merge_parts_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem));
    merge_parts_kernel<<<nq, 256, smem, s>>>(d_ids, d_dist, d_lens, nparts, nq, k_in, k, cap,
                                             d_out_ids, d_out_dist, d_out_len);
    PXC_CUDA(cudaGetLastError());
    ctx->launches += 1;
  });
}

}  // extern "C"
