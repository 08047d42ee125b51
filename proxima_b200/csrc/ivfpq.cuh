// ivfpq.cuh — the IVF-PQ handle, shared by ivfpq.cu (training, parts,
// search) and snapshot.cu (snapshot load and save).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <vector>

#include "common.cuh"

namespace pxc {
namespace ivf {
constexpr uint32_t UNASSIGNED = 0xFFFFFFFFu;  // list_of of a slot in no list (ivfpq.rs UNASSIGNED)
constexpr uint32_t MAX_M = 64;
constexpr uint32_t MAX_DIM = 1024;
}  // namespace ivf
}  // namespace pxc

// ---------------------------------------------------------------------------
// Handle
// ---------------------------------------------------------------------------
struct pxc_ivfpq {
  pxc_ctx* ctx = nullptr;
  uint32_t dim = 0, nlist = 0, m = 0;
  int32_t metric = 0;
  std::vector<uint32_t> widths, offsets;
  pxc::DBuf<uint32_t> woff;
  pxc::DBuf<float> centroids, codebooks, vectors;
  bool have_parts = false, have_vectors = false;
  // u8 re-rank rows: 0 = not built since the store changed, 1 = built, 2 = not applicable
  int u8_state = 0;
  pxc::DBuf<uint8_t> vec_u8;
  pxc::DBuf<int> u8_flag;
  int* h_u8_flag = nullptr;  // pinned
  uint64_t nslots = 0, nlive = 0;
  std::vector<uint64_t> h_ids;
  std::vector<uint8_t> h_live;
  pxc::DBuf<uint64_t> ids;
  pxc::DBuf<uint32_t> slot_rank, rank_slot;
  pxc::DBuf<uint32_t> list_off, list_slot, list_of, list_rank;
  pxc::DBuf<unsigned long long> scanned;
  unsigned long long* h_scanned = nullptr;  // pinned
  pxc::DBuf<uint8_t> list_codes, codes, live;
  bool have_lists = false;
  pxc::DBuf<float> q_buf;
  pxc::DBuf<uint32_t> probes, coarse_d, coarse_len, coarse_zero;
  pxc::DBuf<uint64_t> coarse_l, io_ids, bitmap;
  pxc::DBuf<float> io_dist;
  pxc::DBuf<uint32_t> io_len;
  cudaEvent_t ev_begin = nullptr, ev_end = nullptr;  // scan timing when the context profiles
  bool timed = false;
  cudaEvent_t ev_done = nullptr;  // end of the last search's work (handoff of the scratch)
  std::mutex mu;
  ~pxc_ivfpq() {
    if (ev_done) {
      cudaEventSynchronize(ev_done);  // a search on another stream may still be running
      cudaEventDestroy(ev_done);
    }
    if (h_scanned) cudaFreeHost(h_scanned);
    if (h_u8_flag) cudaFreeHost(h_u8_flag);
    if (ev_begin) cudaEventDestroy(ev_begin);
    if (ev_end) cudaEventDestroy(ev_end);
  }
};


namespace pxc {
namespace ivf {
// ProductQuantizer subspace widths and offsets (product.rs:227-238).
void layout(uint32_t dim, uint32_t m, std::vector<uint32_t>& w, std::vector<uint32_t>& o);
// Waits (host) for the handle's last search before its index is rewritten.
void handoff_drain(pxc_ivfpq* h);
// The list CSR (list_off, list_slot, list_codes, list_rank) on the device
// from per-slot list keys (d_keys: the list of a live assigned slot,
// UNASSIGNED otherwise) and h->codes: a stable sort of the slots by key, so
// every list holds its slots in ascending order. Needs slot_rank. Returns
// once enqueued on `s`.
void build_lists_device(pxc_ivfpq* h, const uint32_t* d_keys, cudaStream_t s);
// slot_rank / rank_slot on the device from the live slots (ascending) and
// their VectorIds, sorted by id. The smallest slot whose id repeats an
// earlier slot's goes to *d_dup (initialised by the caller). Enqueued on `s`.
void rank_ids_device(pxc_ivfpq* h, const uint32_t* d_live_slots, const uint64_t* d_live_ids, uint64_t nlive,
                     uint32_t* d_dup, cudaStream_t s);
// The slot store from host or device vectors (pxc_ivfpq_set_store / _device).
void set_store(pxc_ivfpq* h, const float* vectors, bool on_device, const uint64_t* ids, const uint8_t* live,
               uint64_t nslots);
}  // namespace ivf
}  // namespace pxc
