// select.cuh — block-wide selection over 64-bit keys in shared memory.
#pragma once
#include <stdint.h>

#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>

namespace pxc {

constexpr uint32_t SENTINEL = 0xFFFFFFFFu;  // excluded candidate (filtered / padding)

// Block radix-select: the K-th smallest (1-based) of buf[0, cnt), then keeps
// exactly the K keys <= it at the front (in no particular order). Keys are
// unique. Returns the K-th. hist: 256 words of shared memory, sh: 4.
// Passes of 8 bits from the top; the passes stop as soon as the bin holding
// the K-th is kept whole (then every key of that bin and below is kept, and
// no lower bits need resolving). The kept keys are compacted in place in
// rounds of blockDim keys: each round reads its keys, then writes them down
// to positions no later than any key still unread.
template <uint32_t PER>
__device__ uint64_t select_keep(uint64_t* buf, uint32_t cnt, uint32_t K, uint32_t* hist, uint32_t* sh) {
  __shared__ unsigned long long s_kmax;
  uint64_t prefix = 0, mask = 0, thr = ~0ull;
  uint32_t k = K;
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (uint32_t b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < cnt; i += blockDim.x) {
      const uint64_t key = buf[i];
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) {  // one warp: prefix sums over the 256 bins
      const uint32_t lane = threadIdx.x;
      uint32_t c[8], s = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[lane * 8 + j];
        s += c[j];
      }
      uint32_t inc = s;
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if (lane >= (uint32_t)o) inc += v;
      }
      const uint32_t before = inc - s;
      if (before < k && inc >= k) {
        uint32_t acc = before;
        for (int j = 0; j < 8; ++j) {
          if (acc + c[j] >= k) {
            sh[0] = lane * 8 + j;
            sh[1] = k - acc;
            sh[3] = c[j];
            break;
          }
          acc += c[j];
        }
      }
    }
    __syncthreads();
    const uint32_t bin = sh[0], kr = sh[1], whole = sh[3];
    prefix |= (uint64_t)bin << shift;
    mask |= 0xFFull << shift;
    k = kr;
    __syncthreads();
    if (whole == kr) {  // the K-th is the largest key of its bin: keep the bin whole
      thr = shift == 0 ? prefix : (prefix | ((1ull << shift) - 1ull));
      break;
    }
  }
  if (threadIdx.x == 0) s_kmax = 0;
  uint32_t written = 0;
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  unsigned long long kmax = 0;
  for (uint32_t base = 0; base < cnt; base += blockDim.x) {
    const uint32_t i = base + threadIdx.x;
    const uint64_t key = i < cnt ? buf[i] : ~0ull;
    const bool keep = i < cnt && key <= thr;
    const uint32_t ball = __ballot_sync(0xFFFFFFFFu, keep);
    if (lane == 0) hist[warp] = __popc(ball);
    __syncthreads();  // every key of this round has been read
    uint32_t pos = written + __popc(ball & ((1u << lane) - 1u)), total = 0;
    for (uint32_t w = 0; w < nwarps; ++w) {
      const uint32_t cw = hist[w];
      pos += w < warp ? cw : 0u;
      total += cw;
    }
    if (keep) {
      buf[pos] = key;
      kmax = max(kmax, (unsigned long long)key);
    }
    written += total;
    __syncthreads();  // the counts are read before the next round writes them
  }
  atomicMax(&s_kmax, kmax);
  __syncthreads();
  return s_kmax;
}


// Chunked selection, one block per query. L_in holds the running top-k of
// ranks below c0 as (key << 32 | rank) in ascending RANK order; the chunk adds
// ranks c0.. . The new list is the k smallest of the union under
// (key, rank), written in ascending rank order again, so equal keys resolve
// to the smaller rank. Found with a 4-pass radix select on the key and a
// stable block-wide compaction.
constexpr int SEL_THREADS = 256;
static __global__ void __launch_bounds__(SEL_THREADS) select_chunk_kernel(
    const uint64_t* __restrict__ L_in, const uint32_t* __restrict__ len_in,
    uint64_t* __restrict__ L_out, uint32_t* __restrict__ len_out, const uint32_t* __restrict__ D,
    uint32_t C, uint64_t c0, uint32_t cvalid, uint32_t k, uint32_t q_base) {
  using Scan = cub::BlockScan<uint32_t, SEL_THREADS>;
  using Reduce = cub::BlockReduce<uint32_t, SEL_THREADS>;
  __shared__ typename Scan::TempStorage scan_tmp;
  __shared__ typename Reduce::TempStorage red_tmp;
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_mask, s_remaining, s_take_all, s_thr, s_survivors;
  const uint32_t q = q_base + blockIdx.x;
  const uint64_t* Lq = L_in + (size_t)blockIdx.x * k;
  uint64_t* Oq = L_out + (size_t)blockIdx.x * k;
  const uint32_t* Dq = D + (size_t)q * C;
  const uint32_t lin = len_in[blockIdx.x];
  const uint32_t n = lin + cvalid;

  // Fast path: a full list rejects every chunk key that is not strictly below
  // its worst key (a chunk rank is larger than every listed rank).
  if (lin == k) {
    uint32_t worst = 0;
    for (uint32_t i = threadIdx.x; i < lin; i += SEL_THREADS)
      worst = max(worst, static_cast<uint32_t>(Lq[i] >> 32));
    uint32_t w = Reduce(red_tmp).Reduce(worst, cub::Max());
    if (threadIdx.x == 0) s_thr = w;
    __syncthreads();
    uint32_t cnt = 0;
    for (uint32_t i = threadIdx.x; i < cvalid; i += SEL_THREADS) cnt += Dq[i] < s_thr;
    uint32_t total = Reduce(red_tmp).Sum(cnt);
    if (threadIdx.x == 0) s_survivors = total;
    __syncthreads();
    if (s_survivors == 0) {
      for (uint32_t i = threadIdx.x; i < lin; i += SEL_THREADS) Oq[i] = Lq[i];
      if (threadIdx.x == 0) len_out[blockIdx.x] = lin;
      return;
    }
  }

  auto key_at = [&](uint32_t i) -> uint32_t {
    return i < lin ? static_cast<uint32_t>(Lq[i] >> 32) : Dq[i - lin];
  };
  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_remaining = k;
    s_take_all = 0;
  }
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (uint32_t i = threadIdx.x; i < 256; i += SEL_THREADS) hist[i] = 0;
    __syncthreads();
    if (s_take_all) break;
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (uint32_t i = threadIdx.x; i < n; i += SEL_THREADS) {
      uint32_t key = key_at(i);
      if (key != SENTINEL && (key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t need = s_remaining, cum = 0, digit = 256;
      for (uint32_t b = 0; b < 256; ++b) {
        if (cum + hist[b] >= need) {
          digit = b;
          break;
        }
        cum += hist[b];
      }
      if (digit == 256) {
        s_take_all = 1;  // fewer than `need` candidates share the prefix: all of them fit
      } else {
        s_prefix = prefix | (digit << shift);
        s_mask = mask | (255u << shift);
        s_remaining = need - cum;
      }
    }
    __syncthreads();
  }
  const bool take_all = s_take_all != 0;
  const uint32_t thr = s_prefix, quota_eq = s_remaining;
  // Stable compaction in (list, chunk) = ascending rank order.
  uint32_t out_base = 0, eq_base = 0;
  for (uint32_t base = 0; base < n; base += SEL_THREADS) {
    const uint32_t i = base + threadIdx.x;
    uint32_t key = SENTINEL;
    uint64_t packed = 0;
    if (i < n) {
      if (i < lin) {
        packed = Lq[i];
        key = static_cast<uint32_t>(packed >> 32);
      } else {
        key = Dq[i - lin];
        packed = (static_cast<uint64_t>(key) << 32) | static_cast<uint32_t>(c0 + (i - lin));
      }
    }
    const bool valid = key != SENTINEL;
    uint32_t is_eq = (!take_all && valid && key == thr) ? 1u : 0u;
    uint32_t eq_before, eq_total;
    Scan(scan_tmp).ExclusiveSum(is_eq, eq_before, eq_total);
    __syncthreads();
    bool sel = valid && (take_all || key < thr || (is_eq && eq_base + eq_before < quota_eq));
    uint32_t pos, sel_total;
    Scan(scan_tmp).ExclusiveSum(sel ? 1u : 0u, pos, sel_total);
    __syncthreads();
    if (sel) Oq[out_base + pos] = packed;
    out_base += sel_total;
    eq_base += eq_total;
  }
  if (threadIdx.x == 0) len_out[blockIdx.x] = out_base;
}

}  // namespace pxc
