// hostcopy.cu — the pinned ring and copy threads of hostcopy.cuh.
#include "hostcopy.cuh"

#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace pxc {
namespace hostcopy {

namespace {

constexpr size_t CHUNK = 8u << 20;   // bytes per pinned chunk
constexpr int SLOTS = 4;             // chunks in the ring
constexpr size_t DIRECT = 1u << 20;  // below this a plain cudaMemcpyAsync is as fast

// A memcpy split across a few persistent threads (the caller takes a part too).
class Pool {
 public:
  explicit Pool(int threads) {
    for (int t = 0; t < threads; ++t) workers_.emplace_back([this] { loop(); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> lock(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& w : workers_) w.join();
  }
  void copy(uint8_t* dst, const uint8_t* src, size_t n) {
    const int parts = (int)workers_.size() + 1;
    if (n < (256u << 10) || parts == 1) {
      std::memcpy(dst, src, n);
      return;
    }
    {
      std::lock_guard<std::mutex> lock(mu_);
      dst_ = dst;
      src_ = src;
      n_ = n;
      parts_ = parts;
      next_ = 0;
      left_ = parts;
      ++gen_;
    }
    cv_.notify_all();
    work();
    std::unique_lock<std::mutex> lock(mu_);
    done_.wait(lock, [this] { return left_ == 0; });
  }

 private:
  void work() {  // take parts until none is left
    for (;;) {
      int part;
      uint8_t* d;
      const uint8_t* s;
      size_t n;
      int parts;
      {
        std::lock_guard<std::mutex> lock(mu_);
        if (next_ >= parts_) return;
        part = next_++;
        d = dst_;
        s = src_;
        n = n_;
        parts = parts_;
      }
      const size_t per = ((n + parts - 1) / parts + 63) & ~size_t(63);
      const size_t b = std::min(n, per * part), e = std::min(n, b + per);
      if (e > b) std::memcpy(d + b, s + b, e - b);
      {
        std::lock_guard<std::mutex> lock(mu_);
        if (--left_ == 0) done_.notify_all();
      }
    }
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lock(mu_);
        cv_.wait(lock, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
      }
      work();
    }
  }
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, done_;
  uint8_t* dst_ = nullptr;
  const uint8_t* src_ = nullptr;
  size_t n_ = 0;
  int parts_ = 0, next_ = 0, left_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

struct Stager {
  std::mutex mu;  // one staged copy at a time per context
  uint8_t* ring = nullptr;
  cudaEvent_t ev[SLOTS] = {};
  bool pending[SLOTS] = {};
  Pool pool;
  int device;
  explicit Stager(int dev)
      : pool(std::max(1, std::min(7, (int)std::thread::hardware_concurrency() / 2 - 1))), device(dev) {}
  ~Stager() {
    for (int i = 0; i < SLOTS; ++i)
      if (ev[i]) {
        cudaEventSynchronize(ev[i]);
        cudaEventDestroy(ev[i]);
      }
    if (ring) cudaFreeHost(ring);
  }
  void ensure() {
    if (ring) return;
    PXC_CUDA(cudaMallocHost(&ring, CHUNK * SLOTS));
    for (int i = 0; i < SLOTS; ++i) PXC_CUDA(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming));
  }
  void wait_slot(int i) {
    if (pending[i]) PXC_CUDA(cudaEventSynchronize(ev[i]));
    pending[i] = false;
  }
};

std::mutex g_create_mu;

Stager* stager(pxc_ctx* ctx) {
  std::lock_guard<std::mutex> lock(g_create_mu);
  if (!ctx->stager) {
    ctx->stager = new Stager(ctx->device);
    ctx->stager_free = &release;
  }
  return static_cast<Stager*>(ctx->stager);
}

bool is_pinned(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

}  // namespace

void release(void* p) { delete static_cast<Stager*>(p); }

void to_device(pxc_ctx* ctx, void* dst, const void* src, size_t n, cudaStream_t s) {
  if (!n) return;
  if (n < DIRECT || is_pinned(src)) {
    PXC_CUDA(cudaMemcpyAsync(dst, src, n, cudaMemcpyHostToDevice, s));
    return;
  }
  Stager* st = stager(ctx);
  std::lock_guard<std::mutex> lock(st->mu);
  st->ensure();
  const uint8_t* in = static_cast<const uint8_t*>(src);
  uint8_t* out = static_cast<uint8_t*>(dst);
  int slot = 0;
  for (size_t off = 0; off < n; off += CHUNK, slot = (slot + 1) % SLOTS) {
    const size_t len = std::min(CHUNK, n - off);
    st->wait_slot(slot);  // the copy engine is done with this chunk's last contents
    uint8_t* pin = st->ring + (size_t)slot * CHUNK;
    st->pool.copy(pin, in + off, len);
    PXC_CUDA(cudaMemcpyAsync(out + off, pin, len, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaEventRecord(st->ev[slot], s));
    st->pending[slot] = true;
  }
}

void to_host(pxc_ctx* ctx, void* dst, const void* src, size_t n, cudaStream_t s) {
  if (!n) return;
  if (n < DIRECT || is_pinned(dst)) {
    PXC_CUDA(cudaMemcpyAsync(dst, src, n, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    return;
  }
  Stager* st = stager(ctx);
  std::lock_guard<std::mutex> lock(st->mu);
  st->ensure();
  for (int i = 0; i < SLOTS; ++i) st->wait_slot(i);
  const uint8_t* in = static_cast<const uint8_t*>(src);
  uint8_t* out = static_cast<uint8_t*>(dst);
  const size_t chunks = (n + CHUNK - 1) / CHUNK;
  auto issue = [&](size_t c) {
    const int slot = (int)(c % SLOTS);
    const size_t off = c * CHUNK, len = std::min(CHUNK, n - off);
    PXC_CUDA(cudaMemcpyAsync(st->ring + (size_t)slot * CHUNK, in + off, len, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaEventRecord(st->ev[slot], s));
    st->pending[slot] = true;
  };
  // keep SLOTS - 1 chunks in flight ahead of the one being drained
  for (size_t c = 0; c < std::min<size_t>(chunks, SLOTS - 1); ++c) issue(c);
  for (size_t c = 0; c < chunks; ++c) {
    if (c + SLOTS - 1 < chunks) issue(c + SLOTS - 1);
    const int slot = (int)(c % SLOTS);
    st->wait_slot(slot);
    const size_t off = c * CHUNK, len = std::min(CHUNK, n - off);
    st->pool.copy(out + off, st->ring + (size_t)slot * CHUNK, len);
  }
}

}  // namespace hostcopy
}  // namespace pxc
