// sq_tc.cuh — K12: the scalar-quantized scan's score GEMM on tcgen05 tensor
// cores (kind::i8, s8 x s8 -> s32), with the selection it feeds fused into
// the epilogue.
//
// Operands: A = the queries in code space (s8, 128 per CTA, resident in
// shared memory for the whole pass), B = the I8 codes of the filter-accepted
// rows in ascending rank order ("columns"), streamed 256 rows per tile. The
// s32 result S = sum_c q8_c * code_c is exact integer arithmetic, so every
// kernel configuration produces the same keys; a column's key is
// 0x80000000 - S (ascending key = descending score) and candidates are
// compared as (key << 32 | column), which breaks equal scores toward the
// lower rank.
//
// Two epilogues over the same main loop:
//   DENSE   writes every key of columns [c_begin, c_end) to a query-major
//           matrix (the prefix pass, and the exact fallback);
//   THRESH  appends only the columns whose key is <= the query's admission
//           key tau to a per-query candidate buffer (one reservation per
//           lane per tile). The host derives tau from the prefix pass and
//           checks afterwards that enough columns passed for the result to
//           be exact; a query whose buffer overflows (its count exceeds the
//           capacity) is redone by the host.
//
// Structure: one CTA per 128 queries x one contiguous range of tiles.
//   warp 0      TMA producer: the query tile once (kblocks boxes of 128 B x
//               128 rows), then code tiles (128 B x 256 rows per stage)
//               through a STAGES-deep ring; 128-byte swizzle;
//   warp 1      allocates 512 TMEM columns = two 128 x 256 s32 accumulators
//               and issues tcgen05.mma (M=128, N=256, K=32), alternating
//               accumulators per tile so the epilogue of tile t overlaps the
//               MMAs of tile t+1;
//   warps 2-9   epilogue: TMEM lane quarter (warp & 3) x column half
//               ((warp-2) >> 2), one query row per thread.
// Every mbarrier wait is bounded; on expiry the CTA records DEV_TIMEOUT_* in
// the status word, drains its own copies and MMAs, frees TMEM and returns.
#pragma once
#include "common.cuh"
#include "select.cuh"
#include "sm100.cuh"

namespace pxc {
namespace sq_tc {

constexpr int BM = 128;        // queries per CTA = UMMA M
constexpr int BN = 256;        // code rows per tile = UMMA N
constexpr int KB_BYTES = 128;  // one 128-byte swizzle atom of K per TMA box
constexpr int UMMA_K = 32;     // K bytes per tcgen05.mma kind::i8
constexpr int A_BLOCK = BM * KB_BYTES;  // 16 KiB per K block
constexpr int B_BLOCK = BN * KB_BYTES;  // 32 KiB per stage
constexpr int NUM_EPI_WARPS = 8;
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;  // 320
constexpr int MAX_KBLOCKS = 8;                        // dim <= 1024
constexpr size_t SMEM_LIMIT = 227 * 1024;
constexpr int MODE_DENSE = 0;
constexpr int MODE_THRESH = 1;
constexpr uint32_t HIT_BUF = 8;  // THRESH: admitted columns buffered per thread before a flush

struct Params {
  uint32_t* dense;        // DENSE: [nq_rows][dense_ld] keys of columns c_begin..
  uint64_t dense_ld;
  const uint32_t* tau;    // THRESH: admission key per query
  uint64_t* cand;         // THRESH: [nq_rows][cap] (key << 32 | column)
  uint32_t* cand_cnt;     // THRESH: [nq_rows] appended (may exceed cap: overflow)
  uint32_t cap;
  uint32_t* status;       // device error word
  uint32_t nq;            // valid query rows
  uint32_t c_begin;       // first column of the pass
  uint32_t c_end;         // one past the last valid column
  uint32_t kblocks;       // code pitch / 128
  uint32_t ntiles;        // ceil((c_end - c_begin) / BN)
  uint32_t tiles_per_split;
  uint32_t stages;
  uint64_t wait_ns;
};

__host__ __device__ inline size_t smem_bytes(uint32_t kblocks, uint32_t stages) {
  size_t off = (size_t)kblocks * A_BLOCK + (size_t)stages * B_BLOCK;
  off += (2 * stages + 6) * sizeof(uint64_t) + 16;
  return off + 1024;  // alignment slack
}

// Stages in the ring: as many as fit, at most 8.
__host__ inline uint32_t pick_stages(uint32_t kblocks) {
  const size_t fixed = (size_t)kblocks * A_BLOCK + 1024 + 256;
  const uint32_t s = (uint32_t)((SMEM_LIMIT - fixed) / (B_BLOCK + 16));
  return s > 8 ? 8 : s;
}

__device__ __forceinline__ uint32_t score_key(int32_t s) { return 0x80000000u - static_cast<uint32_t>(s); }

__device__ __forceinline__ void record_failure(uint32_t* status, uint32_t code) {
  if (atomicCAS(status, 0u, code) == 0u) atomicExch(status + 1, blockIdx.y * gridDim.x + blockIdx.x);
}

// v[j] for a lane-varying j without dynamic register indexing (which would
// move v to local memory): a five-level select tree.
__device__ __forceinline__ uint32_t pick32(const uint32_t (&v)[32], uint32_t j) {
  uint32_t a[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = (j & 16) ? v[i + 16] : v[i];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = (j & 8) ? a[i + 8] : a[i];
#pragma unroll
  for (int i = 0; i < 4; ++i) a[i] = (j & 4) ? a[i + 4] : a[i];
  a[0] = (j & 2) ? a[2] : a[0];
  a[1] = (j & 2) ? a[3] : a[1];
  return (j & 1) ? a[1] : a[0];
}

template <int MODE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    sq_scan_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_c,
                   const Params p) {
  using namespace sm100;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t kblocks = p.kblocks, stages = p.stages;
  unsigned char* sA = smem;
  unsigned char* sB = smem + (size_t)kblocks * A_BLOCK;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + (size_t)stages * B_BLOCK);
  uint64_t* full = bars;
  uint64_t* empty = bars + stages;
  uint64_t* acc_full = bars + 2 * stages;  // [2]: one per accumulator
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint64_t* a_full = acc_empty + 2;
  uint64_t* mma_done = a_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  __shared__ volatile uint32_t failed;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t qtile = blockIdx.x, split = blockIdx.y;
  const uint32_t t_begin = split * p.tiles_per_split;
  const uint32_t t_end = min(t_begin + p.tiles_per_split, p.ntiles);
  const uint32_t ntile_local = t_end > t_begin ? t_end - t_begin : 0;

  if (warp == 1) {
    tmem_alloc<512>(tmem_slot);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    failed = 0;
    for (uint32_t s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], NUM_EPI_WARPS * 32);
    }
    mbar_init(a_full, 1);
    mbar_init(mma_done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_c);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0 && ntile_local > 0) {
      mbar_arrive_expect_tx(a_full, kblocks * A_BLOCK);
      for (uint32_t kb = 0; kb < kblocks; ++kb)
        tma_load_2d(sA + (size_t)kb * A_BLOCK, &tmap_q, a_full, kb * KB_BYTES, qtile * BM);
    }
    __syncwarp();
    uint32_t it = 0;
    bool ok = true;
    for (uint32_t t = 0; t < ntile_local && ok; ++t) {
      const int32_t y = static_cast<int32_t>(p.c_begin + (t_begin + t) * BN);
      for (uint32_t kb = 0; kb < kblocks; ++kb, ++it) {
        const uint32_t s = it % stages, ph = (it / stages) & 1;
        const bool fl = failed;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&empty[s], ph ^ 1, p.wait_ns) && !fl)) {
          if (lane == 0) record_failure(p.status, DEV_TIMEOUT_EMPTY);
          failed = 1;
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s], B_BLOCK);
          tma_load_2d(sB + (size_t)s * B_BLOCK, &tmap_c, &full[s], kb * KB_BYTES, y);
        }
        __syncwarp();
      }
    }
    // Drain: every copy this warp issued has landed before the CTA exits.
    const uint32_t first = it > stages ? it - stages : 0;
    for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % stages], (j / stages) & 1, p.wait_ns);
    if (ntile_local > 0) mbar_wait(a_full, 0, p.wait_ns);
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // A: signed 8-bit (bit 7), B: signed 8-bit (bit 10), D: s32.
    const uint32_t idesc = idesc_u8_s32(BM, BN) | (1u << 7) | (1u << 10);
    bool ok = true;
    if (ntile_local > 0) {
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(a_full, 0, p.wait_ns));
      if (!ok) {
        if (lane == 0) record_failure(p.status, DEV_TIMEOUT_FULL);
        failed = 1;
      }
    }
    tc_fence_after();
    const uint32_t a_addr = smem_u32(sA), b_addr = smem_u32(sB);
    uint32_t it = 0;
    for (uint32_t t = 0; t < ntile_local && ok; ++t) {
      const uint32_t b = t & 1, use = t >> 1;
      bool fl = failed;
      // this accumulator was drained by the epilogue (tile t-2)
      if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_empty[b], (use & 1) ^ 1, p.wait_ns) && !fl)) {
        if (lane == 0) record_failure(p.status, DEV_TIMEOUT_ACC);
        failed = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + b * BN;
      for (uint32_t kb = 0; kb < kblocks; ++kb, ++it) {
        const uint32_t s = it % stages, ph = (it / stages) & 1;
        fl = failed;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&full[s], ph, p.wait_ns) && !fl)) {
          if (lane == 0) record_failure(p.status, DEV_TIMEOUT_FULL);
          failed = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint64_t adesc = smem_desc_k_sw128(a_addr + kb * A_BLOCK);
          const uint64_t bdesc = smem_desc_k_sw128(b_addr + s * B_BLOCK);
#pragma unroll
          for (uint32_t k = 0; k < KB_BYTES / UMMA_K; ++k)
            // K advance inside the 128-byte swizzle atom: +32 bytes = +2 in
            // the 16-byte-unit start-address field.
            mma_i8(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
          mma_commit(&empty[s]);  // the stage is free once these MMAs complete
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) mma_commit(&acc_full[b]);
      __syncwarp();
    }
    // All MMAs of this warp complete before TMEM is released.
    if (lane == 0) mma_commit(mma_done);
    __syncwarp();
    mbar_wait(mma_done, 0, p.wait_ns);
  } else {
    // ---------------- epilogue: warps 2..9 ----------------
    const uint32_t ew = warp - 2;
    const uint32_t quarter = warp & 3;    // TMEM lanes this warp may read
    const uint32_t colhalf = ew >> 2;     // which 128 columns of each tile
    const uint32_t row = quarter * 32 + lane;
    const uint32_t q = qtile * BM + row;
    const bool qvalid = q < p.nq;
    int32_t sthr = 0x7FFFFFFF;  // THRESH: emit columns with S >= sthr
    if (MODE == MODE_THRESH && qvalid) {
      const int64_t t = (int64_t)0x80000000ll - (int64_t)p.tau[q];
      sthr = t > 0x7FFFFFFFll ? 0x7FFFFFFF : static_cast<int32_t>(t);
    }
    // THRESH: admitted (key << 32 | column) pairs wait in a small register
    // buffer; a full buffer (and the CTA's end) reserves room with one atomic
    // and stores them, so the epilogue rarely waits on a global atomic.
    uint64_t hb[HIT_BUF];
    uint32_t hn = 0;
    auto flush = [&]() {
      if (hn == 0) return;
      const uint32_t pos = atomicAdd(p.cand_cnt + q, hn);
      uint64_t* dst = p.cand + (size_t)q * p.cap;
#pragma unroll
      for (uint32_t i = 0; i < HIT_BUF; ++i)
        if (i < hn && pos + i < p.cap) dst[pos + i] = hb[i];
      hn = 0;
    };
    for (uint32_t t = 0; t < ntile_local; ++t) {
      const uint32_t b = t & 1, use = t >> 1;
      const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[b], use & 1, p.wait_ns) && !failed);
      if (!ok) {
        record_failure(p.status, DEV_TIMEOUT_ACC);
        failed = 1;
        break;
      }
      tc_fence_after();
      const uint32_t col_tile = p.c_begin + (t_begin + t) * BN + colhalf * 128;
      const uint32_t taddr = tmem_base + ((quarter * 32) << 16) + b * BN + colhalf * 128;
      // two 32-column chunks in flight per wait
#pragma unroll 1
      for (uint32_t c = 0; c < 4; c += 2) {
        uint32_t v[2][32];
        tmem_ld_32x32b_x32(taddr + c * 32, v[0]);
        tmem_ld_32x32b_x32(taddr + (c + 1) * 32, v[1]);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t col0 = col_tile + (c + h) * 32;
          if (MODE == MODE_DENSE) {
            if (qvalid) {
              uint4* dst = reinterpret_cast<uint4*>(p.dense + (size_t)q * p.dense_ld + (col0 - p.c_begin));
#pragma unroll
              for (int j4 = 0; j4 < 8; ++j4) {
                uint32_t k4[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const uint32_t col = col0 + 4 * j4 + u;
                  k4[u] = col < p.c_end ? score_key(static_cast<int32_t>(v[h][4 * j4 + u])) : SENTINEL;
                }
                dst[j4] = make_uint4(k4[0], k4[1], k4[2], k4[3]);
              }
            }
          } else {
            uint32_t m = 0;
#pragma unroll
            for (int j = 0; j < 32; ++j) m |= static_cast<uint32_t>(static_cast<int32_t>(v[h][j]) >= sthr) << j;
            const uint32_t lim = p.c_end > col0 ? min(32u, p.c_end - col0) : 0u;
            if (lim < 32) m &= (1u << lim) - 1u;
            if (!qvalid) m = 0;
            // one admitted column per lane per round, rounds while any lane has one left
            while (__any_sync(0xFFFFFFFFu, m != 0)) {
              if (m) {
                const uint32_t j = __ffs(m) - 1;
                m &= m - 1;
                const uint64_t key = (static_cast<uint64_t>(score_key(static_cast<int32_t>(pick32(v[h], j)))) << 32) |
                                     (col0 + j);
                if (hn == HIT_BUF) flush();
#pragma unroll
                for (uint32_t i = HIT_BUF - 1; i > 0; --i) hb[i] = hb[i - 1];
                hb[0] = key;
                ++hn;
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
    if (MODE == MODE_THRESH) flush();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc<512>(tmem_base);
}

}  // namespace sq_tc
}  // namespace pxc
