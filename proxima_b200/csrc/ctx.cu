// ctx.cu — device context, the NCCL communicator and the multi-GPU
// candidate exchange + merge.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <new>
#include <string>
#include <thread>

#include "common.cuh"
#include "topk.cuh"

namespace pxc {

// NCCL is resolved at run time (dlopen of libnccl.so.2, the copy a process
// such as PyTorch has already loaded, else the system's), so the library
// loads, and single-GPU use works, without it.
struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

static NcclApi load_nccl() {
  NcclApi a;
  void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) {
    a.why = "libnccl.so.2 not found";
    return a;
  }
  auto sym = [&](const char* name) {
    void* p = dlsym(lib, name);
    if (!p && a.why.empty()) a.why = std::string("libnccl lacks ") + name;
    return p;
  };
  a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(sym("ncclGetUniqueId"));
  a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(sym("ncclCommInitRank"));
  a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(sym("ncclCommDestroy"));
  a.comm_abort = reinterpret_cast<decltype(a.comm_abort)>(sym("ncclCommAbort"));
  a.comm_async_error = reinterpret_cast<decltype(a.comm_async_error)>(sym("ncclCommGetAsyncError"));
  a.all_gather = reinterpret_cast<decltype(a.all_gather)>(sym("ncclAllGather"));
  a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(sym("ncclAllReduce"));
  a.send = reinterpret_cast<decltype(a.send)>(sym("ncclSend"));
  a.recv = reinterpret_cast<decltype(a.recv)>(sym("ncclRecv"));
  a.group_start = reinterpret_cast<decltype(a.group_start)>(sym("ncclGroupStart"));
  a.group_end = reinterpret_cast<decltype(a.group_end)>(sym("ncclGroupEnd"));
  a.error_string = reinterpret_cast<decltype(a.error_string)>(sym("ncclGetErrorString"));
  a.ok = a.why.empty();
  return a;
}

static const NcclApi& nccl_api() {
  static const NcclApi api = load_nccl();
  return api;
}

static const NcclApi& nccl() {
  const NcclApi& api = nccl_api();
  if (!api.ok) throw make_failure(PXC_CONFIGURATION, 0, 0, "nccl", "NCCL is unavailable: %s", api.why.c_str());
  return api;
}

#define PXC_NCCL(expr)                                                                           \
  do {                                                                                           \
    ncclResult_t r__ = (expr);                                                                   \
    if (r__ != ncclSuccess)                                                                      \
      throw ::pxc::make_failure(PXC_DEVICE, (uint64_t)r__, 0, "nccl", "%s: %s", #expr,          \
                                ::pxc::nccl().error_string(r__));                              \
  } while (0)

// Waits for the stream with the communicator's timeout; on expiry or an
// asynchronous NCCL error the communicator is aborted (later collectives on
// it fail at once) and PXC_TIMEOUT / PXC_DEVICE is raised.
static void wait_comm(pxc_ctx* ctx, cudaStream_t s, const char* where) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) return;
    if (q != cudaErrorNotReady) PXC_CUDA(q);
    ncclResult_t ae = ncclSuccess;
    if (ctx->comm) nccl().comm_async_error(static_cast<ncclComm_t>(ctx->comm), &ae);
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (ae != ncclSuccess || ms > (long long)ctx->comm_timeout_ms) {
      if (ctx->comm) nccl().comm_abort(static_cast<ncclComm_t>(ctx->comm));
      ctx->comm = nullptr;
      ctx->nranks = 1;
      ctx->rank = 0;
      if (ae != ncclSuccess)
        throw make_failure(PXC_DEVICE, (uint64_t)ae, 0, "nccl", "%s: %s (communicator aborted)", where,
                           nccl().error_string(ae));
      throw make_failure(PXC_TIMEOUT, ctx->comm_timeout_ms, 0, "nccl",
                         "%s: the exchange did not finish within %u ms (communicator aborted)", where,
                         ctx->comm_timeout_ms);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

void comm_allgather(pxc_ctx* ctx, const void* send, void* recv, size_t bytes, cudaStream_t s, const char* where) {
  if (ctx->nranks <= 1 || ctx->comm == nullptr) {
    PXC_CUDA(cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    return;
  }
  PXC_NCCL(nccl().all_gather(send, recv, bytes, ncclUint8, static_cast<ncclComm_t>(ctx->comm), s));
  wait_comm(ctx, s, where);
}

size_t exchange_segment_bytes(uint32_t nq, uint32_t k_in) {
  const size_t raw = (size_t)nq * k_in * 12 + (size_t)nq * 4;
  return (raw + 15) / 16 * 16;
}

unsigned char* exchange_send_buffer(pxc_ctx* ctx, size_t bytes) {
  if (bytes > ctx->x_send_bytes) {
    if (ctx->x_send) cudaFree(ctx->x_send);
    ctx->x_send = nullptr;
    ctx->x_send_bytes = 0;
    PXC_CUDA(cudaMalloc(&ctx->x_send, bytes));
    ctx->x_send_bytes = bytes;
  }
  return ctx->x_send;
}

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
// (total_cmp(distance), id), keep k. Part p's lists start at ids + p *
// stride_ids, dist + p * stride_dist and lens + p * stride_len (elements);
// entry (q, i) at q * k_in + i, the length of q at q.
__global__ void merge_parts_kernel(const uint64_t* __restrict__ ids, const float* __restrict__ dist,
                                   const uint32_t* __restrict__ lens, uint32_t nparts, uint32_t nq,
                                   uint32_t k_in, uint32_t k, uint32_t cap, size_t stride_ids,
                                   size_t stride_dist, size_t stride_len, uint64_t* __restrict__ out_ids,
                                   float* __restrict__ out_dist, uint32_t* __restrict__ out_len) {
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
    uint32_t len = min(lens[p * stride_len + q], k_in);
    for (uint32_t i = threadIdx.x; i < len; i += blockDim.x) {
      uint32_t pos = atomicAdd(&count, 1u);
      const size_t e = (size_t)q * k_in + i;
      skey[pos] = order_key(dist[p * stride_dist + e]);
      sid[pos] = ids[p * stride_ids + e];
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

// Merge of part lists that are each sorted by (total_cmp(distance), id), as
// every search of this library returns them: one warp per query; each
// candidate's output position is its index in its own list plus, per other
// list, the number of entries ahead of it (binary search; an equal entry of a
// lower part counts as ahead), so positions are distinct and no sort is needed.
__device__ __forceinline__ bool entry_before(uint32_t ka, uint64_t ia, uint32_t kb, uint64_t ib) {
  return ka < kb || (ka == kb && ia < ib);
}
__global__ void __launch_bounds__(128) merge_sorted_kernel(const uint64_t* __restrict__ ids,
                                                           const float* __restrict__ dist,
                                                           const uint32_t* __restrict__ lens, uint32_t nparts,
                                                           uint32_t nq, uint32_t k_in, uint32_t k, size_t stride_ids,
                                                           size_t stride_dist, size_t stride_len,
                                                           uint64_t* __restrict__ out_ids, float* __restrict__ out_dist,
                                                           uint32_t* __restrict__ out_len) {
  const uint32_t q = blockIdx.x * 4 + (threadIdx.x >> 5);
  const uint32_t lane = threadIdx.x & 31;
  if (q >= nq) return;
  const size_t row = (size_t)q * k_in;
  uint32_t total = 0;
  for (uint32_t p = 0; p < nparts; ++p) total += min(lens[p * stride_len + q], k_in);
  for (uint32_t c = lane; c < nparts * k_in; c += 32) {
    const uint32_t p = c / k_in, i = c - p * k_in;
    const uint32_t len = min(lens[p * stride_len + q], k_in);
    if (i >= len) continue;
    const uint32_t key = order_key(dist[p * stride_dist + row + i]);
    const uint64_t id = ids[p * stride_ids + row + i];
    uint32_t pos = i;
    for (uint32_t o = 0; o < nparts && pos < k; ++o) {
      if (o == p) continue;
      const uint32_t lo_len = min(lens[o * stride_len + q], k_in);
      // entries of list o ahead of (key, id): strictly before, or equal when o < p
      uint32_t a = 0, b = lo_len;
      while (a < b) {
        const uint32_t mid = (a + b) >> 1;
        const uint32_t km = order_key(dist[o * stride_dist + row + mid]);
        const uint64_t im = ids[o * stride_ids + row + mid];
        const bool ahead = entry_before(km, im, key, id) || (o < p && km == key && im == id);
        if (ahead)
          a = mid + 1;
        else
          b = mid;
      }
      pos += a;
    }
    if (pos < k) {
      out_ids[(size_t)q * k + pos] = id;
      out_dist[(size_t)q * k + pos] = dist[p * stride_dist + row + i];
    }
  }
  if (lane == 0) out_len[q] = min(total, k);
}

// Shared-memory size and launch of the merge for `total` candidates per query.
static void launch_merge(const uint64_t* ids, const float* dist, const uint32_t* lens, uint32_t nparts, uint32_t nq,
                         uint32_t k_in, uint32_t k, size_t stride_ids, size_t stride_dist, size_t stride_len,
                         uint64_t* out_ids, float* out_dist, uint32_t* out_len, cudaStream_t s) {
  const uint64_t total = (uint64_t)nparts * k_in;
  uint32_t cap = 1;
  while (cap < total) cap <<= 1;
  if (cap < 32) cap = 32;
  size_t smem = cap * sizeof(uint32_t) + ((cap * sizeof(uint32_t)) & 4) + cap * sizeof(uint64_t);
  if (smem > 48 * 1024)
    PXC_CUDA(cudaFuncSetAttribute(merge_parts_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  merge_parts_kernel<<<nq, 256, smem, s>>>(ids, dist, lens, nparts, nq, k_in, k, cap, stride_ids, stride_dist,
                                           stride_len, out_ids, out_dist, out_len);
  PXC_CUDA(cudaGetLastError());
}

void exchange_and_merge(pxc_ctx* ctx, const unsigned char* send, uint32_t nq, uint32_t k_in, uint32_t k,
                        uint64_t* d_out_ids, float* d_out_dist, uint32_t* d_out_len, cudaStream_t s) {
  const size_t seg = exchange_segment_bytes(nq, k_in);
  const uint32_t nranks = (uint32_t)ctx->nranks;
  const unsigned char* all = send;
  if (nranks > 1) {
    if ((size_t)nranks * seg > ctx->x_recv_bytes) {
      if (ctx->x_recv) cudaFree(ctx->x_recv);
      ctx->x_recv = nullptr;
      ctx->x_recv_bytes = 0;
      PXC_CUDA(cudaMalloc(&ctx->x_recv, (size_t)nranks * seg));
      ctx->x_recv_bytes = (size_t)nranks * seg;
    }
    PXC_NCCL(nccl().all_gather(send, ctx->x_recv, seg, ncclUint8, static_cast<ncclComm_t>(ctx->comm), s));
    all = ctx->x_recv;
  }
  const uint64_t* ids = reinterpret_cast<const uint64_t*>(all);
  const float* dist = reinterpret_cast<const float*>(all + (size_t)nq * k_in * 8);
  const uint32_t* lens = reinterpret_cast<const uint32_t*>(all + (size_t)nq * k_in * 12);
  // every rank's lists come sorted from its search
  merge_sorted_kernel<<<(nq + 3) / 4, 128, 0, s>>>(ids, dist, lens, nranks, nq, k_in, k, seg / 8, seg / 4, seg / 4,
                                                   d_out_ids, d_out_dist, d_out_len);
  PXC_CUDA(cudaGetLastError());
  ctx->launches += 1;
  wait_comm(ctx, s, "candidate exchange");
}

// Queries [owner_begin(j), owner_begin(j+1)) belong to rank j: an even split.
uint32_t owner_begin(uint32_t nq, uint32_t nranks, uint32_t j) {
  return (uint32_t)(((uint64_t)nq * j) / nranks);
}

// The owner-computes exchange: every rank holds its k_in candidates for all nq
// queries (ids, dist, lens as one search writes them); each rank sends every
// owner only the owner's query slice (three grouped sends per peer) and
// merges the ranks' lists of its own slice.
void exchange_to_owners(pxc_ctx* ctx, const uint64_t* ids, const float* dist, const uint32_t* lens, uint32_t nq,
                        uint32_t k_in, uint32_t k, uint64_t* d_out_ids, float* d_out_dist, uint32_t* d_out_len,
                        cudaStream_t s) {
  const uint32_t nranks = (uint32_t)ctx->nranks, me = (uint32_t)ctx->rank;
  const uint32_t q0 = owner_begin(nq, nranks, me), nmine = owner_begin(nq, nranks, me + 1) - q0;
  const size_t seg = exchange_segment_bytes(nmine, k_in);
  if ((size_t)nranks * seg > ctx->x_recv_bytes) {
    if (ctx->x_recv) cudaFree(ctx->x_recv);
    ctx->x_recv = nullptr;
    ctx->x_recv_bytes = 0;
    PXC_CUDA(cudaMalloc(&ctx->x_recv, (size_t)nranks * seg));
    ctx->x_recv_bytes = (size_t)nranks * seg;
  }
  unsigned char* all = ctx->x_recv;
  const size_t id_off = 0, d_off = (size_t)nmine * k_in * 8, l_off = (size_t)nmine * k_in * 12;
  ncclComm_t comm = static_cast<ncclComm_t>(ctx->comm);
  PXC_NCCL(nccl().group_start());
  for (uint32_t j = 0; j < nranks; ++j) {
    const uint32_t b = owner_begin(nq, nranks, j), n = owner_begin(nq, nranks, j + 1) - b;
    if (n) {
      PXC_NCCL(nccl().send(ids + (size_t)b * k_in, (size_t)n * k_in * 8, ncclUint8, (int)j, comm, s));
      PXC_NCCL(nccl().send(dist + (size_t)b * k_in, (size_t)n * k_in * 4, ncclUint8, (int)j, comm, s));
      PXC_NCCL(nccl().send(lens + b, (size_t)n * 4, ncclUint8, (int)j, comm, s));
    }
    if (nmine) {
      unsigned char* r = all + (size_t)j * seg;
      PXC_NCCL(nccl().recv(r + id_off, (size_t)nmine * k_in * 8, ncclUint8, (int)j, comm, s));
      PXC_NCCL(nccl().recv(r + d_off, (size_t)nmine * k_in * 4, ncclUint8, (int)j, comm, s));
      PXC_NCCL(nccl().recv(r + l_off, (size_t)nmine * 4, ncclUint8, (int)j, comm, s));
    }
  }
  PXC_NCCL(nccl().group_end());
  if (nmine) {
    merge_sorted_kernel<<<(nmine + 3) / 4, 128, 0, s>>>(
        reinterpret_cast<const uint64_t*>(all + id_off), reinterpret_cast<const float*>(all + d_off),
        reinterpret_cast<const uint32_t*>(all + l_off), nranks, nmine, k_in, k, seg / 8, seg / 4, seg / 4, d_out_ids,
        d_out_dist, d_out_len);
    PXC_CUDA(cudaGetLastError());
    ctx->launches += 1;
  }
  wait_comm(ctx, s, "candidate exchange to owners");
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
  if (ctx->comm && nccl_api().ok) nccl_api().comm_destroy(static_cast<ncclComm_t>(ctx->comm));
  if (ctx->x_send) cudaFree(ctx->x_send);
  if (ctx->x_recv) cudaFree(ctx->x_recv);
  if (ctx->stager && ctx->stager_free) ctx->stager_free(ctx->stager);
  if (ctx->crc_tab) cudaFree(ctx->crc_tab);
  if (ctx->crc_scratch) cudaFree(ctx->crc_scratch);
  if (ctx->crc_host) cudaFreeHost(ctx->crc_host);
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
    } else if (std::strcmp(name, "flat_group_sample") == 0) {
      ctx->opt_flat_group_sample = value < 0 ? -1 : value;
    } else if (std::strcmp(name, "flat_collect_cap") == 0) {
      // rounded up to a power of two in [32, 2048]; 0 keeps the group launches
      int64_t cap = 32;
      while (cap < value && cap < 2048) cap <<= 1;
      ctx->opt_flat_collect_cap = value <= 0 ? 0 : cap;
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

pxc_status pxc_comm_unique_id(uint8_t out[128], pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(out != nullptr, "out", 0, "null output");
    ncclUniqueId id;
    PXC_NCCL(nccl().get_unique_id(&id));
    std::memcpy(out, id.internal, sizeof(id.internal));
  });
}

pxc_status pxc_ctx_init_comm(pxc_ctx* ctx, const uint8_t id[128], int32_t nranks, int32_t rank, uint32_t timeout_ms,
                             pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr && id != nullptr, "ctx", 0, "null argument");
    PXC_CONFIG(nranks >= 1 && nranks <= 4096, "nranks", nranks, "must be between 1 and 4096");
    PXC_CONFIG(rank >= 0 && rank < nranks, "rank", rank, "must be in [0, nranks)");
    PXC_CONFIG(timeout_ms >= 100, "timeout_ms", timeout_ms, "must be at least 100");
    std::lock_guard<std::mutex> lock(ctx->comm_mu);
    PXC_CONFIG(ctx->comm == nullptr, "comm", 0, "the context already has a communicator");
    ctx->comm_timeout_ms = timeout_ms;
    if (nranks == 1) {
      ctx->nranks = 1;
      ctx->rank = 0;
      return;
    }
    DeviceGuard g(ctx->device);
    ncclUniqueId uid;
    std::memcpy(uid.internal, id, sizeof(uid.internal));
    ncclComm_t comm = nullptr;
    PXC_NCCL(nccl().comm_init_rank(&comm, nranks, uid, rank));
    ctx->comm = comm;
    ctx->nranks = nranks;
    ctx->rank = rank;
  });
}

int32_t pxc_ctx_comm_size(const pxc_ctx* ctx) { return ctx ? ctx->nranks : 0; }
void pxc_ctx_owned_range(const pxc_ctx* ctx, uint32_t nq, uint32_t* begin, uint32_t* count) {
  const uint32_t nranks = ctx && ctx->nranks > 0 ? (uint32_t)ctx->nranks : 1, me = ctx ? (uint32_t)ctx->rank : 0;
  const uint32_t b = owner_begin(nq, nranks, me);
  if (begin) *begin = b;
  if (count) *count = owner_begin(nq, nranks, me + 1) - b;
}
int32_t pxc_ctx_comm_rank(const pxc_ctx* ctx) { return ctx ? ctx->rank : -1; }

pxc_status pxc_topk_exchange(pxc_ctx* ctx, const uint64_t* d_ids, const float* d_dist, const uint32_t* d_lens,
                             uint32_t nq, uint32_t k_in, uint32_t k, uint64_t* d_out_ids, float* d_out_dist,
                             uint32_t* d_out_len, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(k <= PXC_MAX_K, "k", k, "exceeds the 16777216 result ceiling");
    PXC_CONFIG((uint64_t)ctx->nranks * k_in <= 8192, "nranks*k_in", (uint64_t)ctx->nranks * k_in,
               "the merge holds at most 8192 candidates per query");
    if (nq == 0) return;
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    std::lock_guard<std::mutex> lock(ctx->comm_mu);
    unsigned char* send = exchange_send_buffer(ctx, exchange_segment_bytes(nq, k_in));
    const size_t n = (size_t)nq * k_in;
    PXC_CUDA(cudaMemcpyAsync(send, d_ids, n * 8, cudaMemcpyDeviceToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(send + n * 8, d_dist, n * 4, cudaMemcpyDeviceToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(send + n * 12, d_lens, (size_t)nq * 4, cudaMemcpyDeviceToDevice, s));
    exchange_and_merge(ctx, send, nq, k_in, k, d_out_ids, d_out_dist, d_out_len, s);
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
    launch_merge(d_ids, d_dist, d_lens, nparts, nq, k_in, k, (size_t)nq * k_in, (size_t)nq * k_in, nq, d_out_ids,
                 d_out_dist, d_out_len, s);
    ctx->launches += 1;
  });
}

}  // extern "C"
