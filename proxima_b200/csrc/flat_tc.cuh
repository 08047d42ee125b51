// flat_tc.cuh — K1: exact u8 distance GEMM on tcgen05 tensor cores with a
// fused per-query top-k, for euclidean stores whose rows and queries are
// integers in [0,255].
//
// Why it is exact: for such data every product and every partial sum of the
// reference's squared_euclidean (crates/proxima-core/src/distance.rs:267-283)
// is an integer below 2^24, so the reference's f32 result is the exact
// integer ||q-x||^2 whatever the summation order. The kernel computes q.x
// exactly in s32 (kind::i8, u8 x u8), forms r = ||x||^2 - 2 q.x per column
// and ranks on r; the distance is r + ||q||^2, converted to f32 exactly.
//
// Why ranking on r with a strict '<' is exact: columns are database rows in
// ascending VectorId order ("rank" order), and every thread scans its columns
// in ascending rank, so a later column that ties the current k-th value has a
// larger id and loses the (total_cmp, id) comparison
// (crates/proxima-core/src/topk.rs:63-67).
//
// Structure: one CTA per 256 queries x one contiguous range of database
// rows ("split"), 256 database rows per tile.
//   warp 0      TMA producer: the 256-query tile once, then 256-row database
//               tiles through a STAGES-deep ring (128-byte swizzle);
//   warp 1      allocates all 512 TMEM columns as two 128 x 256 s32
//               accumulators, one per query half; lane 0 issues tcgen05.mma
//               (M=128, N=256, K=32 per instruction). N=256 keeps the
//               shared-memory operand traffic of each MMA at 96 B/clk, so
//               the MMAs and the TMA writes fit the SM's shared-memory port
//               together (with N=128 they serialise and the tile rate halves);
//   warps 2-9   epilogue, one thread per query row (warps 2-5: first query
//               half, 6-9: second): tcgen05.ld 32 columns at a time (two
//               chunks per wait); per chunk a lower bound of r (smallest
//               row term, largest product) against the thread's admission
//               bound, and r = h - 2*dot with a tree min only where some
//               lane cannot rule its chunk out, where a lane with a
//               candidate queues its admitted pairs at once (KT <= 16; with
//               KT = 32 the flagged chunks are re-read from TMEM after the
//               scan instead) for insertion into a sorted register list of
//               KT entries after the accumulator is released.
// Collect mode (COLLECT) keeps no list: the bound stays the caller's T and
// the admitted pairs go to a segment of HBM per (query, split).
// The halves ping-pong: while the tensor core fills one half's accumulator
// for tile t, the other half's epilogue drains tile t-1 (or t).
// The CTAs of one query tile share a per-query bound in global memory (each
// publishes its current k-th r with atomicMin; a candidate strictly above some
// CTA's k-th value cannot be in the global top-k), and a CTA starts from the
// final lists of finished earlier splits of its query tile.
// Every mbarrier wait is bounded by a global-timer limit; on expiry the CTA
// records DEV_TIMEOUT_* in the status word, drains its own copies and MMAs,
// frees TMEM and returns. There is no barrier among the epilogue warps, so a
// warp that gives up cannot strand another.
//
// The same kernel, instantiated with the F16Scan policy, is K2: the screen of
// the tensor-core path for non-integer data and every metric. There the
// operands are f16 copies of the centred rows and queries, each scaled by a
// power of two (exact), the MMA is kind::f16 with f32 accumulation, and the
// epilogue ranks on r = h_x + c_q * (q^ . x^) in f32 (h_x a per-row term, c_q a
// per-query factor that undoes the scales). The lists it returns are screened
// candidates, not answers: the caller re-ranks them exactly and proves each
// query's answer with an error bound on the screen (flat.cu).
#pragma once
#include <type_traits>
#include "common.cuh"
#include "sm100.cuh"

namespace pxc {
namespace flat_tc {

constexpr int BM = 256;        // queries per CTA (two M=128 accumulators)
constexpr int UM = 128;        // UMMA M
constexpr int BN = 256;        // database rows per tile = UMMA N
constexpr int KB_BYTES = 128;  // one 128-byte swizzle atom of K per TMA box
constexpr int UMMA_K = 32;     // K bytes per tcgen05.mma kind::i8
constexpr int A_BLOCK = BM * KB_BYTES;  // 32 KiB per K block
constexpr int B_BLOCK = BN * KB_BYTES;  // 32 KiB per stage
constexpr int NUM_EPI_WARPS = 8;
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;  // 320
constexpr int MAX_KBLOCKS = 2;                        // 256 bytes of K: dim <= 256 (u8), <= 128 (f16)
constexpr int32_t BIG = 0x3FFFFFFF;                   // sentinel: padding columns, empty slots
constexpr uint32_t R_OFFSET = 0x02000000u;            // makes r non-negative for packing
constexpr size_t SMEM_LIMIT = 227 * 1024;
constexpr int MAX_SEEDS = 8;  // finished earlier splits merged into a fresh list

// Instruction descriptor for kind::f16: f16 x f16 -> f32, both K-major
// (PTX ISA instruction-descriptor table).
__host__ __device__ constexpr uint32_t idesc_f16_f32(uint32_t m, uint32_t n) {
  return (1u << 4)     // D format: f32
         | (0u << 7)   // A: f16
         | (0u << 10)  // B: f16
         | ((n >> 3) << 17) | ((m >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// K1: u8 operands, exact s32 products; ranks on r = ||x||^2 - 2 q.x.
struct U8Scan {
  using T = int32_t;
  static constexpr int FIFO_SLOTS = 32;  // deferred-insertion FIFO entries per thread
  __host__ __device__ static constexpr T big() { return BIG; }
  __host__ __device__ static uint32_t pack(T r) { return static_cast<uint32_t>(r) + R_OFFSET; }
  __host__ __device__ static T unpack(uint32_t key) { return static_cast<int32_t>(key - R_OFFSET); }
  __device__ static T next_up(T r) { return r + 1; }
  __device__ static T value(uint32_t acc, T h, float) { return h - 2 * static_cast<int32_t>(acc); }
  // A lower bound of value() over a chunk: the chunk's smallest row term less
  // twice its largest product (the s32 products are non-negative, so their
  // bit patterns order as the f32 values they spell).
  __device__ static T lower_bound(uint32_t vmax_bits, T hmin, float) {
    return hmin - 2 * static_cast<int32_t>(vmax_bits);
  }
  // the value shared as the pruning bound: the list's k-th
  __device__ static T publish(T kth, T, float) { return kth; }
  __device__ static uint32_t idesc() { return sm100::idesc_u8_s32(UM, BN); }
  __device__ static void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    sm100::mma_i8(d, a, b, id, acc);
  }
};

// K2: f16 operands, f32 accumulation; ranks on r = h_x + c_q * (q^ . x^).
struct F16Scan {
  using T = float;
  static constexpr int FIFO_SLOTS = 16;
  __host__ __device__ static constexpr T big() { return 3.0e38f; }
  __host__ __device__ static uint32_t pack(T r) { return order_key(r); }
  __host__ __device__ static T unpack(uint32_t key) { return key_to_float(key); }
  __device__ static T next_up(T r) { return key_to_float(order_key(r) + 1u); }
  __device__ static T value(uint32_t acc, T h, float c) { return fmaf(__uint_as_float(acc), c, h); }
  // A lower bound of value() over a chunk (c < 0 for every metric: it carries
  // the -2 or -1 of the distance): the smallest row term plus c times the
  // largest product; fmaf rounds monotonically, so the bound holds as computed.
  __device__ static T lower_bound(uint32_t vmax_bits, T hmin, float c) {
    return fmaf(__uint_as_float(vmax_bits), c, hmin);
  }
  // the value shared as the pruning bound: the list's last entry, or its k-th
  // plus the query's margin when that is smaller (rows behind it cannot
  // change a provable answer)
  __device__ static T publish(T kth, T last, float delta) { return fminf(last, kth + delta); }
  __device__ static uint32_t idesc() { return idesc_f16_f32(UM, BN); }
  __device__ static void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    mma_f16(d, a, b, id, acc);
  }
};

// per-warp: two tiles of the per-row term and of its per-chunk minima, and
// the deferred-insertion FIFO
constexpr int CHUNKS = BN / 32;
template <class P>
__host__ __device__ constexpr size_t norm_bytes() {
  return (size_t)NUM_EPI_WARPS * (2 * BN * 4 + 2 * CHUNKS * 4 + P::FIFO_SLOTS * 32 * sizeof(uint2));
}

struct Params {
  const void* norms;       // per-rank row term (P::T): ||x||^2 for K1; padding ranks hold P::big()
  const float* qcoef;      // K2: per-query factor c_q (nullptr for K1)
  const float* qdelta;     // K2: per-query margin added to the k-th value before it is shared (nullptr: 0)
  uint32_t* bound;         // [nq_pad] shared pruning bound per query, as a packed key (P::pack)
  uint32_t* done_count;    // [nqt] finished splits per query tile
  uint32_t* done_list;     // [nqt][nsplit] finished split ids in finishing order (~0u = not yet)
  uint64_t* out_part;      // [nq_pad][nsplit][KT] packed P::pack(r)<<32 | rank
  // collect mode only: every (r, rank) with r <= the starting bound, unordered,
  // in one private segment per (query, split)
  uint64_t* cand = nullptr;      // [nq][nsplit][cand_cap] packed P::pack(r)<<32 | rank
  uint32_t* cand_cnt = nullptr;  // [nq][nsplit] entries found (may exceed cand_cap: overflow)
  uint32_t cand_cap = 0;
  // 0: every split keeps its own list (no seeding from finished splits, no
  // shared bound published), so the splits' lists hold disjoint rows
  uint32_t share = 1;
  uint32_t split_stride = 0;  // tiles between the first tiles of consecutive splits (0: tiles_per_split)
  uint32_t* status;        // device error word
  uint32_t nq;
  uint32_t k;              // the list position whose value is shared as the pruning bound (<= KT, see P::publish)
  uint32_t kblocks;        // K bytes / 128
  uint32_t ntiles;         // nrank_pad / BN
  uint32_t tiles_per_split;
  uint32_t nsplit;
  uint32_t stages;
  uint64_t wait_ns;
};

template <class P>
__host__ __device__ inline size_t smem_bytes(uint32_t kblocks, uint32_t stages) {
  size_t off = (size_t)kblocks * A_BLOCK + (size_t)stages * B_BLOCK + norm_bytes<P>();
  off += (2 * stages + 6) * sizeof(uint64_t) + 16;
  return off + 1024;  // alignment slack
}

// Stages in the ring: as many as fit, at most 8.
template <class P>
__host__ inline uint32_t pick_stages(uint32_t kblocks) {
  size_t fixed = (size_t)kblocks * A_BLOCK + norm_bytes<P>() + 1024 + 256;
  uint32_t s = (uint32_t)((SMEM_LIMIT - fixed) / (B_BLOCK + 16));
  return s > 8 ? 8 : s;
}

// Branch-free insertion into an ascending register list; precondition
// r < lr[K-1]. Elements equal to r stay ahead of it (they have smaller ids).
template <int K, class T>
__device__ __forceinline__ void insert_sorted(T (&lr)[K], uint32_t (&lk)[K], T r, uint32_t rank) {
#pragma unroll
  for (int i = K - 1; i > 0; --i) {
    bool shift = lr[i - 1] > r;
    bool here = lr[i] > r;
    T nr = shift ? lr[i - 1] : (here ? r : lr[i]);
    uint32_t nk = shift ? lk[i - 1] : (here ? rank : lk[i]);
    lr[i] = nr;
    lk[i] = nk;
  }
  bool here0 = lr[0] > r;
  lk[0] = here0 ? rank : lk[0];
  lr[0] = here0 ? r : lr[0];
}

__device__ __forceinline__ void record_failure(uint32_t* status, uint32_t code) {
  if (atomicCAS(status, 0u, code) == 0u) atomicExch(status + 1, blockIdx.y * gridDim.x + blockIdx.x);
}

// The shared bound as a value; keys above the sentinel's (the 0xFF.. fill)
// read as the sentinel.
template <class P>
__device__ __forceinline__ typename P::T load_bound(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return P::unpack(min(v, P::pack(P::big())));
}
__device__ __forceinline__ uint32_t load_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void store_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Seed a fresh list with the final lists of up to MAX_SEEDS finished splits
// of the same query tile that cover SMALLER ranks than this split. Their
// entries are real candidates, so the list's k-th value is at once a valid
// and tight admission bound. Exactness is kept: every seeded rank is below
// every rank this split scans, so a scanned column that ties a seeded value
// still loses under the strict '<'; and the seeded entries also remain in
// their own split's list, so the merge (which drops duplicates) sees them.
template <int KT, class P>
__device__ __forceinline__ void seed_from_finished(const Params& p, uint32_t qtile, uint32_t split, uint32_t q,
                                                   typename P::T (&lr)[KT], uint32_t (&lk)[KT]) {
  using T = typename P::T;
  const uint32_t cnt = min(load_acquire(p.done_count + qtile), p.nsplit);
  int used = 0;
  for (uint32_t i = cnt; i > 0 && used < MAX_SEEDS; --i) {
    const uint32_t s2 = load_acquire(p.done_list + (size_t)qtile * p.nsplit + (i - 1));
    if (s2 >= split) continue;  // not yet published, or a later split
    ++used;
    const unsigned long long* src =
        reinterpret_cast<const unsigned long long*>(p.out_part + ((size_t)q * p.nsplit + s2) * KT);
    uint64_t keys[KT];
#pragma unroll
    for (int j = 0; j < KT; ++j) keys[j] = __ldcg(src + j);  // all loads in flight at once
#pragma unroll
    for (int j = 0; j < KT; ++j) {
      const T r = P::unpack(static_cast<uint32_t>(keys[j] >> 32));
      if (!(r < lr[KT - 1])) continue;
      // A finished split's list may already hold entries it seeded from a
      // third split: admit each rank once, or the list (and the bound it
      // publishes) would rest on fewer than KT distinct candidates.
      const uint32_t rank = static_cast<uint32_t>(keys[j]);
      bool dup = false;
#pragma unroll
      for (int i = 0; i < KT; ++i) dup |= lk[i] == rank && lr[i] == r;
      if (!dup) insert_sorted<KT, T>(lr, lk, r, rank);
    }
  }
}

// r of one 32-column chunk (P::value of the accumulator and the row term);
// returns the chunk minimum (tree reduction: depth 5 instead of a 31-long
// dependency chain).
template <class P>
__device__ __forceinline__ typename P::T chunk_r(const uint32_t (&v)[32], const typename P::T* nrm, float c,
                                                 typename P::T (&r)[32]) {
  using T = typename P::T;
#pragma unroll
  for (int j4 = 0; j4 < 8; ++j4) {
    const int4 hb = *reinterpret_cast<const int4*>(nrm + 4 * j4);
    const T h[4] = {*reinterpret_cast<const T*>(&hb.x), *reinterpret_cast<const T*>(&hb.y),
                    *reinterpret_cast<const T*>(&hb.z), *reinterpret_cast<const T*>(&hb.w)};
#pragma unroll
    for (int j = 0; j < 4; ++j) r[4 * j4 + j] = P::value(v[4 * j4 + j], h[j], c);
  }
  T m[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) m[j] = min(r[j], r[j + 16]);
#pragma unroll
  for (int j = 0; j < 8; ++j) m[j] = min(m[j], m[j + 8]);
#pragma unroll
  for (int j = 0; j < 4; ++j) m[j] = min(m[j], m[j + 4]);
  return min(min(m[0], m[2]), min(m[1], m[3]));
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// Bit pattern of the largest of 32 accumulator values read as f32 (a tree of
// three-input maxima).
__device__ __forceinline__ uint32_t chunk_max_bits(const uint32_t (&v)[32]) {
  float m[11];
#pragma unroll
  for (int j = 0; j < 10; ++j)
    m[j] = fmax3(__uint_as_float(v[3 * j]), __uint_as_float(v[3 * j + 1]), __uint_as_float(v[3 * j + 2]));
  m[10] = fmaxf(__uint_as_float(v[30]), __uint_as_float(v[31]));
  const float a = fmax3(m[0], m[1], m[2]), b = fmax3(m[3], m[4], m[5]), c = fmax3(m[6], m[7], m[8]);
  return __float_as_uint(fmax3(fmax3(a, b, c), m[9], m[10]));
}

// Writes one tile's row terms (a: columns 4*lane.., b: 128 + 4*lane..) and
// the minimum of each 32-column chunk into this warp's slot.
template <class P>
__device__ __forceinline__ void stage_norms(typename P::T* slot, typename P::T* slot_min, int4 a, int4 b,
                                            uint32_t lane) {
  using T = typename P::T;
  reinterpret_cast<int4*>(slot)[lane] = a;
  reinterpret_cast<int4*>(slot)[32 + lane] = b;
  const T* x = reinterpret_cast<const T*>(&a);
  const T* y = reinterpret_cast<const T*>(&b);
  T m0 = min(min(x[0], x[1]), min(x[2], x[3]));
  T m1 = min(min(y[0], y[1]), min(y[2], y[3]));
#pragma unroll
  for (int off = 4; off > 0; off >>= 1) {
    m0 = min(m0, __shfl_xor_sync(0xFFFFFFFFu, m0, off));
    m1 = min(m1, __shfl_xor_sync(0xFFFFFFFFu, m1, off));
  }
  if ((lane & 7u) == 0) {
    slot_min[lane >> 3] = m0;
    slot_min[CHUNKS / 2 + (lane >> 3)] = m1;
  }
}

// Minimum of r over one 32-column chunk without keeping r (fast path).
template <class P>
__device__ __forceinline__ typename P::T chunk_min(const uint32_t (&v)[32], const typename P::T* nrm, float c) {
  typename P::T r[32];
  return chunk_r<P>(v, nrm, c, r);
}

// Whether the chunk holds a value below thr for this lane. Most chunks are
// ruled out by the lower bound (about 17 instructions); the exact minimum is
// taken only when some lane of the warp cannot rule its chunk out.
template <class P>
__device__ __forceinline__ bool chunk_hit(const uint32_t (&v)[32], const typename P::T* nrm, typename P::T hmin,
                                          float c, typename P::T thr) {
  const bool maybe = P::lower_bound(chunk_max_bits(v), hmin, c) < thr;
  if (!__any_sync(0xFFFFFFFFu, maybe)) return false;
  return maybe && chunk_min<P>(v, nrm, c) < thr;
}

// Deferred insertion. A flagged chunk's admitted (r, rank) pairs are pushed
// into the thread's FIFO in shared memory ([slot][lane], conflict-free) while
// the accumulator is held; the FIFO is drained into the register list after
// the accumulator is released, so insertions overlap the next tile's MMAs
// instead of stalling them. FIFO order is ascending rank order, so draining
// with the strict '<' keeps the list exact.
// A FIFO takes a flagged chunk in pieces of P::FIFO_SLOTS columns or fewer,
// draining first when the piece's entries would not fit.
//
// In collect mode (COLLECT) the list stays empty and the bound fixed: a drain
// appends the queued pairs to this thread's own segment of candidates in
// global memory instead (a register counter, no atomics; entries past the
// segment's capacity are counted but not written, which the host reads as an
// overflow).
struct Sink {
  uint64_t* dst;  // this (query, split)'s segment (nullptr: padding query)
  uint32_t n;     // entries found so far
  uint32_t cap;
};

template <int KT, class P, bool COLLECT>
__device__ __forceinline__ void fifo_drain(const uint2* fifo, uint32_t& cnt, uint32_t lane,
                                           typename P::T (&lr)[KT], uint32_t (&lk)[KT],
                                           typename P::T shared_bound, Sink& sink) {
  using T = typename P::T;
  if constexpr (COLLECT) {
    if (sink.dst != nullptr) {
      for (uint32_t i = 0; i < cnt && sink.n + i < sink.cap; ++i) {
        const uint2 e = fifo[i * 32 + lane];
        const T r = *reinterpret_cast<const T*>(&e.x);
        sink.dst[sink.n + i] = (static_cast<uint64_t>(P::pack(r)) << 32) | e.y;
      }
    }
    sink.n += cnt;
  } else {
    const T above = P::next_up(shared_bound);  // admit r <= shared_bound
    for (uint32_t i = 0; i < cnt; ++i) {
      const uint2 e = fifo[i * 32 + lane];
      const T r = *reinterpret_cast<const T*>(&e.x);
      if (r < min(lr[KT - 1], above)) insert_sorted<KT, T>(lr, lk, r, e.y);
    }
  }
  cnt = 0;
}

template <int KT, class P, bool COLLECT>
__device__ __forceinline__ void fifo_push_chunk(const typename P::T (&r)[32], typename P::T thr, uint32_t rank0,
                                                uint2* fifo, uint32_t& cnt, uint32_t lane, typename P::T (&lr)[KT],
                                                uint32_t (&lk)[KT], typename P::T shared_bound, Sink& sink) {
  constexpr int PIECE = P::FIFO_SLOTS < 32 ? P::FIFO_SLOTS : 32;
  static_assert(32 % PIECE == 0, "FIFO pieces must tile the chunk");
#pragma unroll
  for (int j0 = 0; j0 < 32; j0 += PIECE) {
    uint32_t mask = 0;
#pragma unroll
    for (int j = 0; j < PIECE; ++j) mask |= (r[j0 + j] < thr ? 1u : 0u) << j;
    if (cnt + __popc(mask) > (uint32_t)P::FIFO_SLOTS)
      fifo_drain<KT, P, COLLECT>(fifo, cnt, lane, lr, lk, shared_bound, sink);
#pragma unroll
    for (int j = 0; j < PIECE; ++j) {
      if (mask & (1u << j)) {
        fifo[cnt * 32 + lane] = make_uint2(*reinterpret_cast<const uint32_t*>(&r[j0 + j]), rank0 + j0 + j);
        ++cnt;
      }
    }
  }
}

// The scan of one chunk with the push inline: ruled out by the lower bound,
// or r is formed once, its minimum taken and, for a lane with a value within
// thr, the admitted pairs queued.
template <int KT, class P, bool COLLECT>
__device__ __forceinline__ void scan_push_chunk(const uint32_t (&v)[32], const typename P::T* nrm, typename P::T hmin,
                                              float c, typename P::T thr, uint32_t rank0, uint2* fifo, uint32_t& cnt,
                                              uint32_t lane, typename P::T (&lr)[KT], uint32_t (&lk)[KT],
                                              typename P::T shared_bound, Sink& sink) {
  const bool maybe = P::lower_bound(chunk_max_bits(v), hmin, c) < thr;
  if (!__any_sync(0xFFFFFFFFu, maybe)) return;
  typename P::T r[32];
  const typename P::T m = chunk_r<P>(v, nrm, c, r);
  if (maybe && m < thr) fifo_push_chunk<KT, P, COLLECT>(r, thr, rank0, fifo, cnt, lane, lr, lk, shared_bound, sink);
}

template <int KT, class P, bool COLLECT = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    flat_scan_kernel(const __grid_constant__ CUtensorMap tmap_q,
                     const __grid_constant__ CUtensorMap tmap_x, const Params p) {
  using namespace sm100;
  using T = typename P::T;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t kblocks = p.kblocks, stages = p.stages;
  unsigned char* sA = smem;
  unsigned char* sB = smem + (size_t)kblocks * A_BLOCK;
  T* sNorm = reinterpret_cast<T*>(sB + (size_t)stages * B_BLOCK);             // [warp][2][BN]
  T* sNormMin = sNorm + NUM_EPI_WARPS * 2 * BN;                               // [warp][2][CHUNKS]
  uint2* sFifo = reinterpret_cast<uint2*>(sNormMin + NUM_EPI_WARPS * 2 * CHUNKS);  // [warp][slot][lane]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sFifo + NUM_EPI_WARPS * P::FIFO_SLOTS * 32);
  uint64_t* full = bars;
  uint64_t* empty = bars + stages;
  uint64_t* acc_full = bars + 2 * stages;  // [2]: one per query half
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint64_t* a_full = acc_empty + 2;
  uint64_t* mma_done = a_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  __shared__ volatile uint32_t failed;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t qtile = blockIdx.x, split = blockIdx.y;
  const uint32_t t_begin = split * (p.split_stride != 0 ? p.split_stride : p.tiles_per_split);
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
    for (int m = 0; m < 2; ++m) {
      mbar_init(&acc_full[m], 1);
      mbar_init(&acc_empty[m], 4 * 32);  // the four epilogue warps of that half
    }
    mbar_init(a_full, 1);
    mbar_init(mma_done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // The producer and MMA roles run as whole, converged warps (every lane
  // waits, lane 0 issues).
  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      mbar_arrive_expect_tx(a_full, kblocks * A_BLOCK);
      for (uint32_t kb = 0; kb < kblocks; ++kb)
        tma_load_2d(sA + (size_t)kb * A_BLOCK, &tmap_q, a_full, kb * KB_BYTES, qtile * BM);
    }
    __syncwarp();
    uint32_t it = 0;
    bool ok = true;
    for (uint32_t t = 0; t < ntile_local && ok; ++t) {
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
          tma_load_2d(sB + (size_t)s * B_BLOCK, &tmap_x, &full[s], kb * KB_BYTES, (t_begin + t) * BN);
        }
        __syncwarp();
      }
    }
    // Drain: every copy this warp issued has landed before the CTA exits.
    const uint32_t first = it > stages ? it - stages : 0;
    for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % stages], (j / stages) & 1, p.wait_ns);
    mbar_wait(a_full, 0, p.wait_ns);
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = P::idesc();
    bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(a_full, 0, p.wait_ns));
    if (!ok) {
      if (lane == 0) record_failure(p.status, DEV_TIMEOUT_FULL);
      failed = 1;
    }
    tc_fence_after();
    const uint32_t a_addr = smem_u32(sA), b_addr = smem_u32(sB);
    for (uint32_t t = 0; t < ntile_local && ok; ++t) {
      const uint32_t it0 = t * kblocks;
      for (uint32_t m = 0; m < 2 && ok; ++m) {
        bool fl = failed;
        // this half's accumulator was drained by its epilogue warps (tile t-1)
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_empty[m], (t & 1) ^ 1, p.wait_ns) && !fl)) {
          if (lane == 0) record_failure(p.status, DEV_TIMEOUT_ACC);
          failed = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        for (uint32_t kb = 0; kb < kblocks; ++kb) {
          const uint32_t it = it0 + kb, s = it % stages, ph = (it / stages) & 1;
          if (m == 0) {
            fl = failed;
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&full[s], ph, p.wait_ns) && !fl)) {
              if (lane == 0) record_failure(p.status, DEV_TIMEOUT_FULL);
              failed = 1;
              ok = false;
              break;
            }
            tc_fence_after();
          }
          if (lane == 0) {
            const uint64_t bdesc = smem_desc_k_sw128(b_addr + s * B_BLOCK);
            const uint64_t adesc = smem_desc_k_sw128(a_addr + kb * A_BLOCK + m * (UM * KB_BYTES));
            const uint32_t d_tmem = tmem_base + m * BN;
#pragma unroll
            for (uint32_t k = 0; k < KB_BYTES / UMMA_K; ++k) {
              // K advance inside the 128-byte swizzle atom: +32 bytes = +2 in
              // the 16-byte-unit start-address field.
              P::mma(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
            }
          }
          __syncwarp();
        }
        if (!ok) break;
        if (lane == 0) mma_commit(&acc_full[m]);
        __syncwarp();
      }
      if (!ok) break;
      // both halves have consumed the tile: release its stages to the producer
      if (lane == 0)
        for (uint32_t kb = 0; kb < kblocks; ++kb) mma_commit(&empty[(it0 + kb) % stages]);
      __syncwarp();
    }
    // All MMAs of this warp complete before TMEM is released.
    if (lane == 0) mma_commit(mma_done);
    __syncwarp();
    mbar_wait(mma_done, 0, p.wait_ns);
  } else {
    // ---------------- epilogue: warps 2..9, one thread per query row ----------------
    const uint32_t ew = warp - 2;
    const uint32_t quarter = warp & 3;
    const uint32_t half = ew >> 2;
    const uint32_t row = half * UM + quarter * 32 + lane;
    const uint32_t q = qtile * BM + row;
    uint32_t* bound_ptr = p.bound + q;
    T* wnorm = sNorm + ew * 2 * BN;  // this warp's two tile slots
    T* wmin = sNormMin + ew * 2 * CHUNKS;
    uint2* wfifo = sFifo + ew * P::FIFO_SLOTS * 32;  // this warp's deferred-insertion FIFO
    uint32_t fifo_cnt = 0;
    const float coef = (p.qcoef != nullptr && q < p.nq) ? p.qcoef[q] : 0.0f;
    const float delta = (p.qdelta != nullptr && q < p.nq) ? p.qdelta[q] : 0.0f;
    T lr[KT];
    uint32_t lk[KT];
#pragma unroll
    for (int i = 0; i < KT; ++i) {
      lr[i] = P::big();
      lk[i] = 0xFFFFFFFFu;
    }
    Sink sink{nullptr, 0, 0};
    if constexpr (COLLECT) {
      if (q < p.nq) sink = Sink{p.cand + ((size_t)q * p.nsplit + split) * p.cand_cap, 0, p.cand_cap};
    } else {
      if (q < p.nq && p.share) seed_from_finished<KT, P>(p, qtile, split, q, lr, lk);
    }
    T shared_bound = load_bound<P>(bound_ptr);  // prune r > shared_bound
    T published = P::big();
    // ||x||^2 of tile t sits in this warp's slot t & 1; tile t+1's is fetched
    // (8 per lane) while tile t is scanned.
    int4 nx0 = make_int4(0, 0, 0, 0), nx1 = nx0;
    if (ntile_local > 0) {
      const int4* src = reinterpret_cast<const int4*>(static_cast<const T*>(p.norms) + (size_t)t_begin * BN);
      stage_norms<P>(wnorm, wmin, __ldg(src + lane), __ldg(src + 32 + lane), lane);
    }
    __syncwarp();
    for (uint32_t t = 0; t < ntile_local; ++t) {
      if (t + 1 < ntile_local) {
        const int4* src = reinterpret_cast<const int4*>(static_cast<const T*>(p.norms) + (size_t)(t_begin + t + 1) * BN);
        nx0 = __ldg(src + lane);
        nx1 = __ldg(src + 32 + lane);
      }
      const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[half], t & 1, p.wait_ns) && !failed);
      if (!ok) {
        record_failure(p.status, DEV_TIMEOUT_ACC);
        failed = 1;
        break;
      }
      tc_fence_after();
      const uint32_t rank_base = (t_begin + t) * BN;
      const uint32_t taddr = tmem_base + ((quarter * 32) << 16) + half * BN;
      const T* nrm = wnorm + (t & 1) * BN;
      const T* nmin = wmin + (t & 1) * CHUNKS;
      // Fast path, branch-free over the whole tile: per chunk only the minimum
      // of r, compared with the admission bound taken at the start of the tile
      // (the list does not change within a tile: insertions are deferred).
      const T thr = min(lr[KT - 1], P::next_up(shared_bound));
      // the other splits' bound is read now and folded in after the tile, so
      // the load's latency hides behind the scan
      const T fresh_bound = load_bound<P>(bound_ptr);
      uint32_t va[32], vb[32];
      uint32_t hit = 0;  // bit c: chunk c holds a candidate for this lane
      if constexpr (COLLECT || (std::is_same<P, U8Scan>::value && KT <= 16)) {
        // A chunk's admitted pairs are queued from the values its exact minimum
        // was taken on instead of re-reading the chunk after the scan (K1 with
        // lists of up to 16 entries, and collect mode, which flags far more
        // chunks: its bound sits near the 800th row). Longer lists keep the
        // re-read: their registers do not leave room for it.
#pragma unroll 1
        for (uint32_t c = 0; c < BN / 32; c += 2) {
          tmem_ld_32x32b_x32(taddr + c * 32, va);
          tmem_ld_32x32b_x32(taddr + (c + 1) * 32, vb);
          tmem_ld_wait();
          scan_push_chunk<KT, P, COLLECT>(va, nrm + c * 32, nmin[c], coef, thr, rank_base + c * 32, wfifo, fifo_cnt, lane, lr,
                               lk, shared_bound, sink);
          scan_push_chunk<KT, P, COLLECT>(vb, nrm + (c + 1) * 32, nmin[c + 1], coef, thr, rank_base + (c + 1) * 32, wfifo,
                               fifo_cnt, lane, lr, lk, shared_bound, sink);
        }
      } else {
#pragma unroll 1
        for (uint32_t c = 0; c < BN / 32; c += 2) {
          // two chunks per wait: the read latency, not the arithmetic, bounds
          // this loop (and nothing runs while a read is in flight)
          tmem_ld_32x32b_x32(taddr + c * 32, va);
          tmem_ld_32x32b_x32(taddr + (c + 1) * 32, vb);
          tmem_ld_wait();
          hit |= static_cast<uint32_t>(chunk_hit<P>(va, nrm + c * 32, nmin[c], coef, thr)) << c;
          hit |= static_cast<uint32_t>(chunk_hit<P>(vb, nrm + (c + 1) * 32, nmin[c + 1], coef, thr)) << (c + 1);
        }
      }
      // Flagged chunks (one vote per tile) are re-read from TMEM and their
      // admitted pairs queued in rank order; the accumulator is released right
      // after. With lists of up to 10 entries two chunks are read per wait;
      // longer lists leave registers for one.
      uint32_t uhit = __reduce_or_sync(0xFFFFFFFFu, hit);
      while (uhit) {
        const uint32_t ca = __ffs(uhit) - 1;
        uhit &= uhit - 1;
        uint32_t cb = BN / 32;
        tmem_ld_32x32b_x32(taddr + ca * 32, va);
        if constexpr (KT <= 10) {
          if (uhit) {
            cb = __ffs(uhit) - 1;
            uhit &= uhit - 1;
            tmem_ld_32x32b_x32(taddr + cb * 32, vb);
          }
        }
        tmem_ld_wait();
        {
          T r[32];
          chunk_r<P>(va, nrm + ca * 32, coef, r);
          fifo_push_chunk<KT, P, COLLECT>(r, thr, rank_base + ca * 32, wfifo, fifo_cnt, lane, lr, lk, shared_bound,
                                          sink);
        }
        if (cb < BN / 32) {
          T r[32];
          chunk_r<P>(vb, nrm + cb * 32, coef, r);
          fifo_push_chunk<KT, P, COLLECT>(r, thr, rank_base + cb * 32, wfifo, fifo_cnt, lane, lr, lk, shared_bound,
                                          sink);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[half]);
      // This warp finished reading slot (t+1)&1 during tile t-1.
      if (t + 1 < ntile_local) stage_norms<P>(wnorm + ((t + 1) & 1) * BN, wmin + ((t + 1) & 1) * CHUNKS, nx0, nx1, lane);
      // insertions happen while the tensor core fills the next tile
      if (fifo_cnt) fifo_drain<KT, P, COLLECT>(wfifo, fifo_cnt, lane, lr, lk, shared_bound, sink);
      __syncwarp();
      // Share the bound with the other splits of this query tile: the k-th
      // value of this split's list (k <= KT, selected without dynamic indexing).
      T kth = lr[KT - 1];
#pragma unroll
      for (int i = 0; i < KT; ++i) kth = (i + 1 == (int)p.k) ? lr[i] : kth;
      const T pub = P::publish(kth, lr[KT - 1], delta);
      if (pub < published && p.share) {
        published = pub;
        atomicMin(bound_ptr, P::pack(published));
      }
      shared_bound = min(shared_bound, fresh_bound);
    }
    if (COLLECT && q < p.nq) p.cand_cnt[(size_t)q * p.nsplit + split] = sink.n;
    if (!COLLECT && q < p.nq) {
      uint64_t* dst = p.out_part + ((size_t)q * p.nsplit + split) * KT;
#pragma unroll
      for (int i = 0; i < KT; ++i)
        dst[i] = (static_cast<uint64_t>(P::pack(lr[i])) << 32) | lk[i];
      __threadfence();  // the list is visible device-wide before this split is announced
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc<512>(tmem_base);
  if (threadIdx.x == 0 && !failed) {
    // Announce the finished split so later splits of this query tile can seed from it.
    __threadfence();
    const uint32_t slot = atomicAdd(p.done_count + qtile, 1u);
    if (slot < p.nsplit) store_release(p.done_list + (size_t)qtile * p.nsplit + slot, split);
  }
}

}  // namespace flat_tc
}  // namespace pxc
