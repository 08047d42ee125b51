// common.cuh — shared definitions of libproxima_cuda.so: status/error
// plumbing, the (total_cmp, id) ordering keys, and the device context.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "proxima_cuda.h"

namespace pxc {

// ---------------------------------------------------------------------------
// Errors. Every entry point catches everything at the boundary and reports
// through pxc_error; nothing throws across the C ABI.
// ---------------------------------------------------------------------------
struct Failure {
  pxc_status code;
  uint64_t a = 0, b = 0;
  char parameter[32] = {0};
  char detail[256] = {0};
};

inline Failure make_failure(pxc_status code, uint64_t a, uint64_t b, const char* parameter,
                            const char* fmt, ...) {
  Failure f;
  f.code = code;
  f.a = a;
  f.b = b;
  if (parameter) std::snprintf(f.parameter, sizeof(f.parameter), "%s", parameter);
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(f.detail, sizeof(f.detail), fmt, ap);
  va_end(ap);
  return f;
}

inline pxc_status report(const Failure& f, pxc_error* err) {
  if (err) {
    err->code = f.code;
    err->a = f.a;
    err->b = f.b;
    std::memcpy(err->parameter, f.parameter, sizeof(err->parameter));
    std::memcpy(err->detail, f.detail, sizeof(err->detail));
  }
  return f.code;
}

inline pxc_status ok(pxc_error* err) {
  if (err) std::memset(err, 0, sizeof(*err));
  return PXC_OK;
}

#define PXC_CUDA(expr)                                                                      \
  do {                                                                                      \
    cudaError_t e__ = (expr);                                                               \
    if (e__ != cudaSuccess)                                                                 \
      throw ::pxc::make_failure(PXC_DEVICE, (uint64_t)e__, 0, nullptr, "%s at %s:%d: %s",   \
                                #expr, __FILE__, __LINE__, cudaGetErrorString(e__));        \
  } while (0)

#define PXC_CONFIG(cond, param, value, reason)                                              \
  do {                                                                                      \
    if (!(cond))                                                                            \
      throw ::pxc::make_failure(PXC_CONFIGURATION, (uint64_t)(value), 0, param, "%s",       \
                                reason);                                                    \
  } while (0)

// Wrap an entry point body: converts Failure and any other exception.
template <class F>
pxc_status guarded(pxc_error* err, F&& body) {
  try {
    body();
    return ok(err);
  } catch (const Failure& f) {
    return report(f, err);
  } catch (const std::exception& e) {
    return report(make_failure(PXC_INTERNAL, 0, 0, nullptr, "%s", e.what()), err);
  } catch (...) {
    return report(make_failure(PXC_INTERNAL, 0, 0, nullptr, "unknown exception"), err);
  }
}

// ---------------------------------------------------------------------------
// Ordering. SearchResult orders by f32::total_cmp then VectorId
// (crates/proxima-core/src/topk.rs:63-67). total_cmp is the signed-integer
// order of the bits after flipping the magnitude of negatives; the unsigned
// form below maps it onto plain u32 order so (key << 32 | rank) compares as
// one u64 when rank follows id order.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t order_key(float f) {
  uint32_t b;
#ifdef __CUDA_ARCH__
  b = __float_as_uint(f);
#else
  std::memcpy(&b, &f, 4);
#endif
  return b ^ ((b & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
}

__host__ __device__ __forceinline__ float key_to_float(uint32_t k) {
  uint32_t b = k ^ ((k & 0x80000000u) ? 0x80000000u : 0xFFFFFFFFu);
#ifdef __CUDA_ARCH__
  return __uint_as_float(b);
#else
  float f;
  std::memcpy(&f, &b, 4);
  return f;
#endif
}

// Device error word written by kernels with bounded waits.
enum DeviceError : uint32_t {
  DEV_OK = 0,
  DEV_TIMEOUT_FULL = 1,
  DEV_TIMEOUT_EMPTY = 2,
  DEV_TIMEOUT_ACC = 3,
  DEV_BAD_SHAPE = 4,
};

}  // namespace pxc

// ---------------------------------------------------------------------------
// Context: one device, one default stream, a small device error/status area.
// ---------------------------------------------------------------------------
struct pxc_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  uint32_t wait_ms = 2000;
  uint32_t* d_status = nullptr;  // [0] device error word, [1] aux
  uint32_t* h_status = nullptr;  // pinned mirror
  int sm_count = 0;
  bool profiling = false;
  unsigned long long launches = 0;  // kernels launched by this library on this context
  std::mutex mu;  // serialises use of the context stream and d_status (k-means, SQ)
  // Diagnostic knobs set through pxc_ctx_set_option (tests only; defaults below).
  int64_t opt_sq_candidate_cap = -1;  // >= 0: shrink the SQ threshold-pass buffers (forces the fallback)
  int64_t opt_sq_spec_rank = -1;      // >= 1: force the SQ speculative admission rank
  bool opt_kmeans_exact = false;      // k-means assignment without the tensor-core screen
  bool opt_kmeans_trace = false;      // k-means prints per-iteration counters to stderr
  int64_t opt_flat_group_sample = -1;  // grouped K1: 1/n of the rows sampled for the bound (-1: 800/k, 0: none)
  int64_t opt_flat_collect_cap = 2048;  // grouped K1: collect-mode slots per query (0: the group launches)
  // k-means scratch kept between calls (grown on demand, freed with the context)
  void* kmeans_ws = nullptr;
  void (*kmeans_ws_free)(void*) = nullptr;
  // The NCCL communicator over the ranks of one job (one context per rank;
  // pxc_ctx_init_comm). Collectives are issued in call order under comm_mu.
  void* comm = nullptr;  // ncclComm_t
  int nranks = 1, rank = 0;
  uint32_t comm_timeout_ms = 60000;
  std::mutex comm_mu;
  unsigned char* x_send = nullptr;  // exchange buffers (device), grown on demand
  unsigned char* x_recv = nullptr;
  size_t x_send_bytes = 0, x_recv_bytes = 0;
  // CRC-32C tables on the device (slicing tables and shift operators),
  // uploaded on first use.
  uint32_t* crc_tab = nullptr;
  uint32_t* crc_scratch = nullptr;  // block values + result of pxc_crc32c_device (device)
  uint32_t* crc_host = nullptr;     // its result (pinned)
  std::mutex crc_mu;
  // pinned ring and copy threads for pageable host <-> device copies (hostcopy.cuh)
  void* stager = nullptr;
  void (*stager_free)(void*) = nullptr;
};

namespace pxc {
// RAII device selection.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) PXC_CUDA(cudaSetDevice(dev));
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Device buffer with RAII free.
template <class T>
struct DBuf {
  T* p = nullptr;
  size_t n = 0;
  DBuf() = default;
  DBuf(const DBuf&) = delete;
  DBuf& operator=(const DBuf&) = delete;
  ~DBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
  void reserve(size_t count) {  // grows, keeps nothing
    if (count <= n) return;
    release();
    if (count == 0) return;
    PXC_CUDA(cudaMalloc(&p, count * sizeof(T)));
    n = count;
  }
  void grow_keep(size_t count, size_t keep, cudaStream_t s) {  // grows, keeps first `keep`
    if (count <= n) return;
    T* q = nullptr;
    PXC_CUDA(cudaMalloc(&q, count * sizeof(T)));
    if (p && keep) PXC_CUDA(cudaMemcpyAsync(q, p, keep * sizeof(T), cudaMemcpyDeviceToDevice, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    if (p) cudaFree(p);
    p = q;
    n = count;
  }
};

// Reads the device error word after a kernel with bounded waits and turns it
// into a Failure. Synchronises the stream.
void check_device_status(pxc_ctx* ctx, cudaStream_t s, const char* where);
// Same for an error word owned by a handle (d_status device, h_status pinned).
void check_status_word(uint32_t* d_status, uint32_t* h_status, cudaStream_t s, const char* where);

// Candidate exchange over the context's communicator: `send` holds this
// rank's segment (ids [nq][k_in] u64 | distances [nq][k_in] f32 | lengths [nq]
// u32, seg_bytes long, 16-byte multiple); one NCCL allgather of the segments,
// then the (total_cmp, id) merge of every rank's lists into the outputs. Waits
// (bounded by the context's communicator timeout) for the work to finish.
size_t exchange_segment_bytes(uint32_t nq, uint32_t k_in);
void exchange_and_merge(pxc_ctx* ctx, const unsigned char* send, uint32_t nq, uint32_t k_in, uint32_t k,
                        uint64_t* d_out_ids, float* d_out_dist, uint32_t* d_out_len, cudaStream_t s);
// The context's send buffer, grown to at least `bytes` (callers hold comm_mu).
unsigned char* exchange_send_buffer(pxc_ctx* ctx, size_t bytes);
uint32_t owner_begin(uint32_t nq, uint32_t nranks, uint32_t j);
void exchange_to_owners(pxc_ctx* ctx, const uint64_t* ids, const float* dist, const uint32_t* lens, uint32_t nq,
                        uint32_t k_in, uint32_t k, uint64_t* d_out_ids, float* d_out_dist, uint32_t* d_out_len,
                        cudaStream_t s);
// ncclAllGather of `bytes` per rank over the context's communicator (recv:
// nranks * bytes, rank order), then the bounded wait of the exchange. With one
// rank, a device copy. Callers hold comm_mu.
void comm_allgather(pxc_ctx* ctx, const void* send, void* recv, size_t bytes, cudaStream_t s, const char* where);
}  // namespace pxc
