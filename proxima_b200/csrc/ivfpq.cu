// ivfpq.cu — IvfPqIndex on the device (crates/proxima-index/src/ivfpq.rs),
// search equal to the reference's search_prepared (:998-1110) on the same
// parts: the same probed lists, scores, shortlist and reranked top-k.
//
// Device layout (HBM):
//   centroids   nlist x dim f32 (coarse quantizer)
//   codebooks   256 x dim f32, subspace-major as ProductQuantizer stores them
//               (subspace s at 256 * offsets[s], entry j at + j * width[s])
//   lists       CSR over lists: list_off[nlist+1]; list_slot[] the live slots
//               of each list in ascending slot order; list_codes[] their PQ
//               codes copied into list order so a list scan reads one
//               contiguous run (16 bytes per code at m = 16)
//   store       vectors (slot-major, prepared), ids, and a rank of every live
//               slot's VectorId, so (score, rank) orders exactly as the
//               reference's (total_cmp(score), id)
//
// Search (per batch of queries):
//   K4 coarse   every centroid's squared_euclidean in the reference's 8-lane
//               order (proxima_core::distance, unrolled) from the tiled fp32
//               distance kernel, top-nprobe by (distance, list index) with a
//               block radix select per query.
//   K5 scan     one CTA per query: for each probed list, the residual table
//               (q - c) against every codebook entry (sequential sums, as
//               ProductQuantizer::distance_table) in shared memory, then the
//               list's codes scored by table lookups (sequential over
//               subspaces, as DistanceTable::squared_l2), kept in a
//               thresholded candidate buffer reduced by a block radix-select;
//   K6 rerank   the shortlist rescored with space.distance on the stored
//               vectors, top-k.
// Cosine uses the query's own table once and 1 - q.c + table.inner_product.
#include <cub/cub.cuh>

#include <algorithm>
#include <cmath>
#include <numeric>
#include <vector>

#include "common.cuh"
#include "hostcopy.cuh"
#include "ivfpq.cuh"
#include "kmeans_api.h"
#include "rng.h"
#include "refdist.cuh"
#include "select.cuh"
#include "fp32scan.cuh"
#include "topk.cuh"

namespace pxc {
namespace ivf {

constexpr uint32_t MAX_NPROBE = 128;
constexpr uint32_t MAX_SHORTLIST = 4096;
constexpr uint32_t SCAN_THREADS = 256;
constexpr uint32_t CB_MAX = 8192; // candidate buffer per query (shared memory), largest
constexpr uint32_t CHUNK = 1024;  // codes scored between buffer checks

// VectorSpace::distance for the two metrics search_prepared scores:
// cosine = 1 - dot_unrolled, euclidean = squared_euclidean.
__device__ __forceinline__ float space_distance(int metric, const float* a, const float* __restrict__ b,
                                                uint32_t dim) {
  return metric == PXC_COSINE ? __fsub_rn(1.0f, dot_unrolled(a, b, dim)) : l2_unrolled(a, b, dim);
}

// The same sums for dim % 8 == 0, two rows at once, each row read as two
// 16-byte loads per group of eight elements (the operation order is
// unchanged: lane l still takes elements l, l+8, ...; the tail of an
// 8-multiple is exactly 0.0 and is still added).
__device__ __forceinline__ void space_distance_vec8x2(int metric, const float* a, const float* __restrict__ b0,
                                                      const float* __restrict__ b1, uint32_t dim, float& d0,
                                                      float& d1) {
  float acc0[8], acc1[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) acc0[l] = acc1[l] = 0.0f;
  const float4* p0 = reinterpret_cast<const float4*>(b0);
  const float4* p1 = reinterpret_cast<const float4*>(b1);
  const bool cosine = metric == PXC_COSINE;
#pragma unroll 2
  for (uint32_t i = 0; i < dim; i += 8) {
    const float4 u0 = __ldg(p0 + i / 4), w0 = __ldg(p0 + i / 4 + 1);
    const float4 u1 = __ldg(p1 + i / 4), w1 = __ldg(p1 + i / 4 + 1);
    const float x0[8] = {u0.x, u0.y, u0.z, u0.w, w0.x, w0.y, w0.z, w0.w};
    const float x1[8] = {u1.x, u1.y, u1.z, u1.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      const float q = a[i + l];
      if (cosine) {
        acc0[l] = __fadd_rn(acc0[l], __fmul_rn(q, x0[l]));
        acc1[l] = __fadd_rn(acc1[l], __fmul_rn(q, x1[l]));
      } else {
        const float e0 = __fsub_rn(q, x0[l]), e1 = __fsub_rn(q, x1[l]);
        acc0[l] = __fadd_rn(acc0[l], __fmul_rn(e0, e0));
        acc1[l] = __fadd_rn(acc1[l], __fmul_rn(e1, e1));
      }
    }
  }
  auto fin = [&](const float (&acc)[8]) {
    const float s0 = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
    const float s1 = __fadd_rn(__fadd_rn(acc[4], acc[5]), __fadd_rn(acc[6], acc[7]));
    const float sum = __fadd_rn(__fadd_rn(s0, s1), 0.0f);
    return cosine ? __fsub_rn(1.0f, sum) : sum;
  };
  d0 = fin(acc0);
  d1 = fin(acc1);
}

// ---------------------------------------------------------------------------
// K4: coarse top-nprobe. The exact 8-lane squared_euclidean of every (query,
// centroid) pair (nearest_centroid's order, ivfpq.rs:1231-1249) comes from the
// tiled fp32 distance kernel as order keys, one row per query; a block-wide
// radix select keeps the nprobe smallest (key, list) per query and this kernel
// sorts them ascending into the probe list (UNASSIGNED past the end).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) probes_from_lists_kernel(const uint64_t* __restrict__ L,
                                                                const uint32_t* __restrict__ len, uint32_t P,
                                                                uint32_t nprobe, uint32_t* __restrict__ probes) {
  __shared__ uint64_t keys[MAX_NPROBE];
  const uint32_t q = blockIdx.x;
  const uint32_t n = min(len[q], P);
  uint32_t n2 = 1;
  while (n2 < n) n2 <<= 1;
  for (uint32_t i = threadIdx.x; i < n2; i += blockDim.x) keys[i] = i < n ? L[(size_t)q * P + i] : ~0ull;
  block_bitonic_sort_u64(keys, n2);
  for (uint32_t i = threadIdx.x; i < nprobe; i += blockDim.x)
    probes[(size_t)q * nprobe + i] = i < n ? static_cast<uint32_t>(keys[i]) : UNASSIGNED;
}

// Re-rank on u8 rows. When the metric is euclidean, dim <= 256 and the query
// and every live row are integers in [0,255], each term (q - x)^2 <= 65025 and
// every partial sum <= 256 * 65025 < 2^24 is an integer, so the reference's
// f32 squared_euclidean is exact in any order and equals the integer sum
// below (|q - x| per byte, then a 4-way dot product of the differences).
constexpr uint32_t U8_MAX_DIM = 256;

__device__ __forceinline__ uint32_t sqdiff_u8x16(const uint4 a, const uint4 b, uint32_t acc) {
  uint32_t d = __vabsdiffu4(a.x, b.x);
  acc = __dp4a(d, d, acc);
  d = __vabsdiffu4(a.y, b.y);
  acc = __dp4a(d, d, acc);
  d = __vabsdiffu4(a.z, b.z);
  acc = __dp4a(d, d, acc);
  d = __vabsdiffu4(a.w, b.w);
  return __dp4a(d, d, acc);
}

struct ScanParams {
  const float* queries;      // nq x dim (prepared)
  const uint32_t* probes;    // nq x nprobe list indices
  const float* centroids;
  const float* codebooks;
  const uint32_t* woff;      // [m] widths then [m+1] offsets
  const uint32_t* list_off;
  const uint32_t* list_slot;
  const uint8_t* list_codes;
  const uint32_t* list_rank;  // VectorId rank of each list entry (list order)
  const uint32_t* rank_slot;
  const uint64_t* ids;        // VectorId per slot
  const float* vectors;       // nullable: no rerank
  const uint8_t* vec_u8;      // nullable: rank-major u8 copy of the live rows (see build_u8_rows)
  const uint64_t* bitmap;     // nullable
  uint64_t* out_ids;
  float* out_dist;
  uint32_t* out_len;
  unsigned long long* scanned;  // codes scored, summed over queries
  uint32_t nq, dim, m, nprobe, k, shortlist;
  uint32_t cb;  // candidate buffer entries (>= shortlist + 2 * CHUNK, >= 4096, <= CB_MAX)
  int metric;
  int rerank;
};

// u8 copy of the live rows in rank order for the u8 re-rank; clears *all_int
// when a component is not an integer in [0,255] (the copy is then unused).
__global__ void build_u8_rows_kernel(const float* __restrict__ vectors, const uint32_t* __restrict__ rank_slot,
                                     uint64_t nrank, uint32_t dim, uint8_t* __restrict__ out,
                                     int* __restrict__ all_int) {
  const uint64_t r = blockIdx.x;
  if (r >= nrank) return;
  const float* row = vectors + (size_t)rank_slot[r] * dim;
  for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) {
    const float v = row[d];
    const bool ok = v >= 0.0f && v <= 255.0f && v == floorf(v);
    if (!ok) *all_int = 0;
    out[r * dim + d] = ok ? static_cast<uint8_t>(v) : 0;
  }
}

// K5 + K6: one CTA per query.
__global__ void __launch_bounds__(SCAN_THREADS) scan_kernel(const ScanParams p) {
  extern __shared__ __align__(16) unsigned char sm_raw[];
  const uint32_t CB = p.cb;
  uint64_t* buf = reinterpret_cast<uint64_t*>(sm_raw);  // [CB]
  float* lut = reinterpret_cast<float*>(buf + CB);      // [m][256]
  float* qs = lut + (size_t)p.m * 256;                  // [dim]
  float* rs = qs + p.dim;                               // [dim]
  uint32_t* woff = reinterpret_cast<uint32_t*>(rs + p.dim);  // [2m+1]
  __shared__ uint32_t hist[256], sh[4], count;
  __shared__ uint64_t thr;
  __shared__ float qdc;
  __shared__ __align__(16) uint8_t qu8[U8_MAX_DIM];  // the query as u8 (u8 re-rank)
  const uint32_t q = blockIdx.x, t = threadIdx.x;
  const uint32_t dim = p.dim, m = p.m;
  const bool cosine = p.metric == PXC_COSINE;
  int q_int = 1;
  for (uint32_t i = t; i < dim; i += blockDim.x) {
    const float v = p.queries[(size_t)q * dim + i];
    qs[i] = v;
    const bool ok = v >= 0.0f && v <= 255.0f && v == floorf(v);
    q_int &= ok ? 1 : 0;
    if (i < U8_MAX_DIM) qu8[i] = ok ? static_cast<uint8_t>(v) : 0;
  }
  for (uint32_t i = t; i < 2 * m + 1; i += blockDim.x) woff[i] = p.woff[i];
  if (t == 0) {
    count = 0;
    thr = ~0ull;
  }
  // the host sets vec_u8 only for euclidean stores of integer rows with dim <= 256, dim % 16 == 0
  const bool rerank_u8 = __syncthreads_and(q_int) && p.vec_u8 != nullptr;
  const uint32_t* widths = woff;
  const uint32_t* offs = woff + m;
  // table over a vector v (in shared memory): squared (or dot) per entry
  auto build_table = [&](const float* v, bool dot) {
    if (dim == 8 * m && (m & 3) == 0) {
      // every subspace 8 wide (C4's layout): four subspaces at a time, four
      // independent chains per thread; each entry keeps its own sequential order
      for (uint32_t s = 0; s < m; s += 4) {
        float4 c[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4* cb = reinterpret_cast<const float4*>(p.codebooks + 256u * (8u * (s + i)) + t * 8u);
          c[i][0] = __ldg(cb);
          c[i][1] = __ldg(cb + 1);
        }
        float4 xv[4][2];  // the vector's 32 components of these subspaces (broadcast reads)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          xv[i][0] = reinterpret_cast<const float4*>(v + 8u * (s + i))[0];
          xv[i][1] = reinterpret_cast<const float4*>(v + 8u * (s + i))[1];
        }
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (uint32_t j = 0; j < 8; ++j) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 h = c[i][j >> 2];
            const float cj = (j & 3) == 0 ? h.x : (j & 3) == 1 ? h.y : (j & 3) == 2 ? h.z : h.w;
            const float4 g = xv[i][j >> 2];
            const float x = (j & 3) == 0 ? g.x : (j & 3) == 1 ? g.y : (j & 3) == 2 ? g.z : g.w;
            if (dot) {
              acc[i] = __fadd_rn(acc[i], __fmul_rn(x, cj));
            } else {
              const float d = __fsub_rn(x, cj);
              acc[i] = __fadd_rn(acc[i], __fmul_rn(d, d));
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) lut[(s + i) * 256 + t] = acc[i];
      }
      return;
    }
    for (uint32_t s = 0; s < m; ++s) {
      const uint32_t w = widths[s], o = offs[s];
      const float* cb = p.codebooks + 256u * o + t * w;
      float acc = 0.0f;
      if (w == 8) {  // the common layout: the codeword in two 16-byte loads, the sum in order
        const float4 c0 = __ldg(reinterpret_cast<const float4*>(cb));
        const float4 c1 = __ldg(reinterpret_cast<const float4*>(cb) + 1);
        const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
        for (uint32_t j = 0; j < 8; ++j) {
          if (dot) {
            acc = __fadd_rn(acc, __fmul_rn(v[o + j], c[j]));
          } else {
            const float d = __fsub_rn(v[o + j], c[j]);
            acc = __fadd_rn(acc, __fmul_rn(d, d));
          }
        }
        lut[s * 256 + t] = acc;
        continue;
      }
      for (uint32_t j = 0; j < w; ++j) {
        const float c = __ldg(cb + j);
        if (dot) {
          acc = __fadd_rn(acc, __fmul_rn(v[o + j], c));
        } else {
          const float d = __fsub_rn(v[o + j], c);
          acc = __fadd_rn(acc, __fmul_rn(d, d));
        }
      }
      lut[s * 256 + t] = acc;
    }
  };
  if (cosine) build_table(qs, true);  // one table per query (the dot products)
  for (uint32_t pi = 0; pi < p.nprobe; ++pi) {
    const uint32_t l = p.probes[(size_t)q * p.nprobe + pi];
    if (l == UNASSIGNED) break;
    const float* c = p.centroids + (size_t)l * dim;
    __syncthreads();  // previous list's lookups are done
    if (!cosine) {
      for (uint32_t i = t; i < dim; i += blockDim.x) rs[i] = __fsub_rn(qs[i], c[i]);
      __syncthreads();
      build_table(rs, false);
    } else if (t == 0) {
      qdc = dot_unrolled(qs, c, dim);
    }
    __syncthreads();
    const float one_minus = cosine ? __fsub_rn(1.0f, qdc) : 0.0f;
    const uint32_t b = p.list_off[l], e = p.list_off[l + 1];
    if (t == 0 && p.scanned) atomicAdd(p.scanned, (unsigned long long)(e - b));
    // m = 16 (one 16-byte code per row): the next chunk's codes are loaded
    // while the current chunk's are looked up
    constexpr int U = CHUNK / SCAN_THREADS;
    uint4 pre[U];
    auto fetch16 = [&](uint32_t j0f) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t j = j0f + t + u * SCAN_THREADS;
        pre[u] = j < e ? __ldg(reinterpret_cast<const uint4*>(p.list_codes) + j) : make_uint4(0u, 0u, 0u, 0u);
      }
    };
    if (m == 16) fetch16(b);
    for (uint32_t j0 = b; j0 < e; j0 += CHUNK) {
      if (count > CB - CHUNK) {
        const uint64_t kth = select_keep<CB_MAX / SCAN_THREADS>(buf, count, p.shortlist, hist, sh);
        if (t == 0) {
          count = p.shortlist;
          thr = kth;
        }
        __syncthreads();
      }
      const uint64_t th = thr;
      const uint32_t j1 = min(e, j0 + CHUNK);
      // four codes per thread at once: four independent lookup chains
      uint4 cur[U];
#pragma unroll
      for (int u = 0; u < U; ++u) cur[u] = pre[u];
      if (m == 16 && j0 + CHUNK < e) fetch16(j0 + CHUNK);
      uint32_t jj[U];
      bool on[U];
      float sum[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        jj[u] = j0 + t + u * SCAN_THREADS;
        on[u] = jj[u] < j1;
        sum[u] = 0.0f;
        if (on[u] && p.bitmap) {
          const uint32_t slot = p.list_slot[jj[u]];
          on[u] = (p.bitmap[slot >> 6] >> (slot & 63)) & 1ull;
        }
      }
      if (m == 16) {
#pragma unroll
        for (int b = 0; b < 16; ++b) {
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const uint32_t word = (b >> 2) == 0 ? cur[u].x : (b >> 2) == 1 ? cur[u].y : (b >> 2) == 2 ? cur[u].z : cur[u].w;
            // byte b & 3 of the word, zero-extended (one PRMT); rows switched off
            // by the filter add their table entries and are dropped at admission
            const uint32_t idx = __byte_perm(word, 0u, 0x4440u + (b & 3));
            sum[u] = __fadd_rn(sum[u], lut[b * 256 + idx]);
          }
        }
      } else if ((m & 15) == 0) {
        for (uint32_t s0 = 0; s0 < m; s0 += 16) {
          uint32_t w4[U][4];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (on[u]) v = __ldg(reinterpret_cast<const uint4*>(p.list_codes + (size_t)jj[u] * m + s0));
            w4[u][0] = v.x, w4[u][1] = v.y, w4[u][2] = v.z, w4[u][3] = v.w;
          }
          const float* rows = lut + s0 * 256;
#pragma unroll
          for (int b = 0; b < 16; ++b) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
              // byte b & 3 of the word, zero-extended (one PRMT)
              const uint32_t idx = __byte_perm(w4[u][b >> 2], 0u, 0x4440u + (b & 3));
              sum[u] = __fadd_rn(sum[u], rows[b * 256 + idx]);
            }
          }
        }
      } else {
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (on[u]) {
            const uint8_t* code = p.list_codes + (size_t)jj[u] * m;
            for (uint32_t s2 = 0; s2 < m; ++s2) sum[u] = __fadd_rn(sum[u], lut[s2 * 256 + code[s2]]);
          }
      }
      // Admission: the score's order key decides alone unless it ties the
      // threshold's, so the rank is loaded only for codes that may enter; one
      // shared-memory reservation per warp and code slot.
      const uint32_t th_hi = static_cast<uint32_t>(th >> 32);
      const uint32_t lane = t & 31;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const float score = cosine ? __fadd_rn(one_minus, -sum[u]) : sum[u];
        const uint32_t ok = order_key(score);
        bool want = on[u] && ok <= th_hi;
        uint64_t key = 0;
        if (want) {
          key = ((uint64_t)ok << 32) | p.list_rank[jj[u]];
          want = key < th;
        }
        const uint32_t mask = __ballot_sync(0xFFFFFFFFu, want);
        if (mask) {
          const uint32_t leader = __ffs(mask) - 1;
          uint32_t base = 0;
          if (lane == leader) base = atomicAdd(&count, static_cast<uint32_t>(__popc(mask)));
          base = __shfl_sync(0xFFFFFFFFu, base, leader);
          if (want) buf[base + __popc(mask & ((1u << lane) - 1u))] = key;
        }
      }
      __syncthreads();
    }
  }
  __syncthreads();
  uint32_t n = count;
  if (n > p.shortlist) {
    select_keep<CB_MAX / SCAN_THREADS>(buf, n, p.shortlist, hist, sh);
    n = p.shortlist;
  }
  uint32_t n2 = 1;
  while (n2 < n) n2 <<= 1;
  for (uint32_t i = n + t; i < n2; i += blockDim.x) buf[i] = ~0ull;
  if (!(p.rerank && p.vectors)) block_bitonic_sort_u64(buf, n2);
  uint64_t* outk = buf;
  if (p.rerank && p.vectors) {
    // (in place: the thread that reads entry i writes its new key to entry i)
    // K6: exact distances of the shortlist, top-k of them
    if (rerank_u8) {
      // 128-byte rows for C4's dim 128: a quarter of the f32 rows' traffic
      const uint32_t nv = dim / 16;
      const uint4* q4 = reinterpret_cast<const uint4*>(qu8);
      for (uint32_t i = t; i < n; i += 2 * blockDim.x) {
        const uint32_t i1 = i + blockDim.x;
        const uint32_t r0 = (uint32_t)buf[i];
        const uint32_t r1 = i1 < n ? (uint32_t)buf[i1] : r0;
        const uint4* x0 = reinterpret_cast<const uint4*>(p.vec_u8 + (size_t)r0 * dim);
        const uint4* x1 = reinterpret_cast<const uint4*>(p.vec_u8 + (size_t)r1 * dim);
        uint32_t a0 = 0, a1 = 0;
#pragma unroll 8
        for (uint32_t j = 0; j < nv; ++j) {
          const uint4 u = __ldg(x0 + j), w = __ldg(x1 + j);
          const uint4 qv = q4[j];
          a0 = sqdiff_u8x16(qv, u, a0);
          a1 = sqdiff_u8x16(qv, w, a1);
        }
        buf[i] = ((uint64_t)order_key(static_cast<float>(a0)) << 32) | r0;
        if (i1 < n) buf[i1] = ((uint64_t)order_key(static_cast<float>(a1)) << 32) | r1;
      }
    } else if ((dim & 7) == 0) {
      // two rows per thread at a time: twice the loads in flight
      for (uint32_t i = t; i < n; i += 2 * blockDim.x) {
        const uint32_t i1 = i + blockDim.x;
        const uint32_t r0 = (uint32_t)buf[i];
        const uint32_t r1 = i1 < n ? (uint32_t)buf[i1] : r0;
        float d0, d1;
        space_distance_vec8x2(p.metric, qs, p.vectors + (size_t)p.rank_slot[r0] * dim,
                              p.vectors + (size_t)p.rank_slot[r1] * dim, dim, d0, d1);
        buf[i] = ((uint64_t)order_key(d0) << 32) | r0;
        if (i1 < n) buf[i1] = ((uint64_t)order_key(d1) << 32) | r1;
      }
    } else {
      for (uint32_t i = t; i < n; i += blockDim.x) {
        const uint32_t rank = (uint32_t)buf[i];
        const float d = space_distance(p.metric, qs, p.vectors + (size_t)p.rank_slot[rank] * dim, dim);
        buf[i] = ((uint64_t)order_key(d) << 32) | rank;
      }
    }
    block_bitonic_sort_u64(buf, n2);
  }
  const uint32_t take = min(n, p.k);
  for (uint32_t i = t; i < take; i += blockDim.x) {
    const uint64_t key = outk[i];
    const uint32_t slot = p.rank_slot[(uint32_t)key];
    p.out_ids[(size_t)q * p.k + i] = p.ids[slot];
    p.out_dist[(size_t)q * p.k + i] = key_to_float((uint32_t)(key >> 32));
  }
  if (t == 0) p.out_len[q] = take;
}

// ---------------------------------------------------------------------------
// Build side: PQ encoding of residuals (ProductQuantizer::encode_into,
// product.rs:361-380 with nearest_centroid :529-547: residual x - c per
// dimension, then the codeword with the smallest sequential squared distance,
// strict '<' so ties keep the lower index). Block = 128 rows x one subspace;
// the subspace's codebook in shared memory, each row's residual too.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) pq_encode_kernel(const float* __restrict__ X, uint32_t ldx, uint64_t n,
                                                        const uint32_t* __restrict__ list_of,
                                                        const float* __restrict__ centroids, uint32_t dim,
                                                        const float* __restrict__ codebooks,
                                                        const uint32_t* __restrict__ woff, uint32_t m,
                                                        uint8_t* __restrict__ codes) {
  extern __shared__ __align__(16) float sm[];
  const uint32_t s = blockIdx.y;
  const uint32_t w = woff[s], o = woff[m + s];
  float* book = sm;              // [256][w]
  float* res = sm + 256 * w;     // [128][w + 1]
  for (uint32_t e = threadIdx.x; e < 256 * w; e += blockDim.x) book[e] = codebooks[256u * o + e];
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  // list_of == nullptr: plain ProductQuantizer::encode_into, the row itself
  const bool valid = i < n && (list_of == nullptr || list_of[i] != UNASSIGNED);
  if (valid) {
    const float* x = X + i * ldx + o;
    if (list_of) {
      const float* c = centroids + (size_t)list_of[i] * dim + o;
      for (uint32_t t = 0; t < w; ++t) res[threadIdx.x * (w + 1) + t] = __fsub_rn(x[t], c[t]);
    } else {
      for (uint32_t t = 0; t < w; ++t) res[threadIdx.x * (w + 1) + t] = x[t];
    }
  }
  __syncthreads();
  if (!valid) {
    if (i < n) codes[i * m + s] = 0;
    return;
  }
  const float* r = res + threadIdx.x * (w + 1);
  uint32_t best = 0;
  float bd = __int_as_float(0x7f800000);
  for (uint32_t j = 0; j < 256; ++j) {
    const float* cw = book + j * w;
    float acc = 0.0f;
    for (uint32_t t = 0; t < w; ++t) {
      const float d = __fsub_rn(r[t], cw[t]);
      acc = __fadd_rn(acc, __fmul_rn(d, d));
    }
    if (acc < bd) {
      bd = acc;
      best = j;
    }
  }
  codes[i * m + s] = (uint8_t)best;
}

// ProductQuantizer::distance_table (product.rs:407-439): for every (query,
// subspace, codeword) the sequential sums l2 += d*d, ip += q*c over the
// subspace width, from 0.0, without contraction. Block = one (query,
// subspace), thread = codeword; out[(q*m + s)*256 + c].
__global__ void __launch_bounds__(256) pq_tables_kernel(const float* __restrict__ Q, uint32_t dim,
                                                        const float* __restrict__ codebooks,
                                                        const uint32_t* __restrict__ woff, uint32_t m,
                                                        float* __restrict__ sq, float* __restrict__ dot) {
  const uint32_t q = blockIdx.x, s = blockIdx.y, c = threadIdx.x;
  const uint32_t w = woff[s], o = woff[m + s];
  const float* qs = Q + (size_t)q * dim + o;
  const float* cw = codebooks + 256ull * o + (size_t)c * w;
  float l2 = 0.0f, ip = 0.0f;
  for (uint32_t t = 0; t < w; ++t) {
    const float qv = __ldg(qs + t), cv = __ldg(cw + t);
    const float d = __fsub_rn(qv, cv);
    l2 = __fadd_rn(l2, __fmul_rn(d, d));
    ip = __fadd_rn(ip, __fmul_rn(qv, cv));
  }
  const size_t e = ((size_t)q * m + s) * 256 + c;
  sq[e] = l2;
  dot[e] = ip;
}

// ProductQuantizer::decode (product.rs:387-398): the chosen codewords, concatenated.
__global__ void pq_decode_kernel(const uint8_t* __restrict__ codes, uint64_t n, uint32_t dim, uint32_t m,
                                 const float* __restrict__ codebooks, const uint32_t* __restrict__ woff,
                                 float* __restrict__ out) {
  const uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (e >= n * m) return;
  const uint64_t i = e / m;
  const uint32_t s = (uint32_t)(e - i * m);
  const uint32_t w = woff[s], o = woff[m + s];
  const float* src = codebooks + 256ull * o + (size_t)codes[e] * w;
  for (uint32_t t = 0; t < w; ++t) out[i * dim + o + t] = src[t];
}

// First non-finite element of n x dim rows (flat index), ~0 if none.
__global__ void first_nonfinite_kernel(const float* __restrict__ X, uint64_t count,
                                       unsigned long long* __restrict__ first) {
  for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < count;
       e += (uint64_t)gridDim.x * blockDim.x)
    if (!isfinite(X[e])) atomicMin(first, (unsigned long long)e);
}

// Residuals of rows against their lists (ivfpq.rs:788-792): x - c per dimension.
__global__ void residual_kernel(const float* __restrict__ X, uint32_t ldx, uint64_t n, uint32_t dim,
                                const uint32_t* __restrict__ list_of, const float* __restrict__ centroids,
                                float* __restrict__ out) {
  const uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (e >= n * dim) return;
  const uint64_t i = e / dim, t = e - i * dim;
  out[e] = __fsub_rn(X[i * ldx + t], centroids[(size_t)list_of[i] * dim + t]);
}

// Gathers rows by index into a dense matrix; and one subspace's columns.
__global__ void gather_rows_kernel(const float* __restrict__ X, uint32_t dim, const uint32_t* __restrict__ rows,
                                   uint64_t n, float* __restrict__ out) {
  const uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (e >= n * dim) return;
  const uint64_t i = e / dim, t = e - i * dim;
  out[e] = X[(size_t)rows[i] * dim + t];
}
__global__ void gather_cols_kernel(const float* __restrict__ X, uint32_t dim, uint64_t n, uint32_t o, uint32_t w,
                                   uint32_t ldo, float* __restrict__ out) {
  const uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (e >= n * w) return;
  const uint64_t i = e / w, t = e - i * w;
  out[i * ldo + t] = X[i * dim + o + t];
}

// Id rank of each list entry, in list order.
__global__ void list_rank_kernel(const uint32_t* __restrict__ list_slot, const uint32_t* __restrict__ slot_rank,
                                 uint64_t n, uint32_t* __restrict__ out) {
  const uint64_t j = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (j < n) out[j] = slot_rank[list_slot[j]];
}

// slot_rank / rank_slot from the live slots sorted by (VectorId, slot): the
// smallest slot whose id repeats an earlier slot's id goes to *dup.
__global__ void rank_ids_kernel(const uint64_t* __restrict__ sorted_ids, const uint32_t* __restrict__ rank_slot,
                                uint64_t nlive, uint32_t* __restrict__ slot_rank, uint32_t* __restrict__ dup) {
  const uint64_t r = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (r >= nlive) return;
  const uint32_t slot = rank_slot[r];
  slot_rank[slot] = (uint32_t)r;
  if (r > 0 && sorted_ids[r] == sorted_ids[r - 1]) atomicMin(dup, slot);
}

// Dead slots take no list.
__global__ void mask_dead_kernel(uint32_t* __restrict__ list_of, const uint8_t* __restrict__ live, uint64_t n) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i < n && !live[i]) list_of[i] = UNASSIGNED;
}
__global__ void iota_u32_kernel(uint32_t* out, uint64_t n) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i < n) out[i] = (uint32_t)i;
}
// List boundaries in the (list, slot)-sorted order.
__global__ void list_bounds_kernel(const uint32_t* __restrict__ keys, uint64_t n, uint32_t nlist,
                                   uint32_t* __restrict__ off) {
  const uint32_t l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l > nlist) return;
  uint64_t lo = 0, hi = n;
  while (lo < hi) {
    const uint64_t mid = (lo + hi) >> 1;
    if (keys[mid] < l)
      lo = mid + 1;
    else
      hi = mid;
  }
  off[l] = (uint32_t)lo;
}
__global__ void gather_codes_kernel(const uint8_t* __restrict__ codes, uint32_t m, const uint32_t* __restrict__ slots,
                                    uint64_t n, uint8_t* __restrict__ out) {
  const uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (e >= n * m) return;
  const uint64_t j = e / m, s = e - j * m;
  out[e] = codes[(size_t)slots[j] * m + s];
}

}  // namespace ivf
}  // namespace pxc

namespace pxc {
namespace ivf {

// The handle's device scratch and index pass from one call to the next in
// stream order. A device search returns once its kernels are enqueued and
// concurrent searches may run on different streams, so each search makes its
// stream wait (on the GPU) for the previous search's work and records the end
// of its own; calls that rewrite the index wait on the host.
void handoff_wait(pxc_ivfpq* h, cudaStream_t s) {
  if (h->ev_done) PXC_CUDA(cudaStreamWaitEvent(s, h->ev_done, 0));
}
void handoff_done(pxc_ivfpq* h, cudaStream_t s) {
  if (!h->ev_done) PXC_CUDA(cudaEventCreateWithFlags(&h->ev_done, cudaEventDisableTiming));
  PXC_CUDA(cudaEventRecord(h->ev_done, s));
}
void handoff_drain(pxc_ivfpq* h) {
  if (h->ev_done) PXC_CUDA(cudaEventSynchronize(h->ev_done));
}

void layout(uint32_t dim, uint32_t m, std::vector<uint32_t>& w, std::vector<uint32_t>& o) {
  // product.rs:227-238 — widths differ by at most one, the remainder leading
  w.assign(m, dim / m);
  for (uint32_t s = 0; s < dim % m; ++s) ++w[s];
  o.assign(m + 1, 0);
  for (uint32_t s = 0; s < m; ++s) o[s + 1] = o[s] + w[s];
}

// Builds the list CSR (ascending slots per list) from list_of and the codes.
void build_lists(pxc_ivfpq* h, const std::vector<uint32_t>& list_of, const uint8_t* codes_host, cudaStream_t s) {
  std::vector<uint32_t> off(h->nlist + 1, 0);
  for (uint64_t i = 0; i < h->nslots; ++i)
    if (h->h_live[i] && list_of[i] != UNASSIGNED) {
      if (list_of[i] >= h->nlist)
        throw make_failure(PXC_CORRUPTION, i, list_of[i], "list_of", "slot %llu names list %u of %u",
                           (unsigned long long)i, list_of[i], h->nlist);
      ++off[list_of[i] + 1];
    }
  for (uint32_t l = 0; l < h->nlist; ++l) off[l + 1] += off[l];
  const uint64_t total = off[h->nlist];
  std::vector<uint32_t> slot(total), fill(off.begin(), off.end() - 1);
  std::vector<uint8_t> lc(std::max<uint64_t>(1, total * h->m));
  for (uint64_t i = 0; i < h->nslots; ++i)
    if (h->h_live[i] && list_of[i] != UNASSIGNED) {
      const uint32_t pos = fill[list_of[i]]++;
      slot[pos] = (uint32_t)i;
      std::memcpy(lc.data() + (size_t)pos * h->m, codes_host + i * h->m, h->m);
    }
  h->list_off.reserve(h->nlist + 1);
  h->list_slot.reserve(std::max<uint64_t>(1, total));
  h->list_codes.reserve(std::max<uint64_t>(16, total * h->m));
  PXC_CUDA(cudaMemcpyAsync(h->list_off.p, off.data(), off.size() * 4, cudaMemcpyHostToDevice, s));
  if (total) {
    PXC_CUDA(cudaMemcpyAsync(h->list_slot.p, slot.data(), total * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(h->list_codes.p, lc.data(), total * h->m, cudaMemcpyHostToDevice, s));
  }
  h->list_rank.reserve(std::max<uint64_t>(1, total));
  if (total)
    list_rank_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(h->list_slot.p, h->slot_rank.p, total,
                                                                      h->list_rank.p);
  PXC_CUDA(cudaStreamSynchronize(s));
  h->have_lists = true;
}

void search_device(pxc_ivfpq* h, const float* d_q, uint32_t nq, uint32_t k, uint32_t nprobe, uint32_t rerank,
                   const uint64_t* d_bitmap, uint64_t* d_ids, float* d_dist, uint32_t* d_len, cudaStream_t s) {
  pxc_ctx* ctx = h->ctx;
  if (nq == 0) return;
  if (k == 0 || h->nlive == 0 || !h->have_lists) {
    PXC_CUDA(cudaMemsetAsync(d_len, 0, (size_t)nq * 4, s));
    return;
  }
  PXC_CONFIG(h->have_parts, "codebooks", 0, "the index has no trained parts");
  nprobe = std::min<uint32_t>(std::max<uint32_t>(nprobe, 1), h->nlist);
  PXC_CONFIG(nprobe <= MAX_NPROBE, "nprobe", nprobe, "the device search supports nprobe <= 128");
  const uint32_t shortlist = rerank > 0 ? std::max(rerank, k) : k;
  PXC_CONFIG(shortlist <= MAX_SHORTLIST, "rerank", shortlist,
             "the device search keeps at most 4096 candidates per query (max(rerank, k))");
  const uint32_t dim = h->dim, nlist = h->nlist;
  if (rerank > 0 && h->have_vectors && h->u8_state == 0) {
    h->u8_state = 2;
    if (h->metric == PXC_EUCLIDEAN && dim <= U8_MAX_DIM && dim % 16 == 0 && h->nlive < (1ull << 31)) {
      h->vec_u8.reserve(h->nlive * dim);
      h->u8_flag.reserve(1);
      if (!h->h_u8_flag) PXC_CUDA(cudaMallocHost(&h->h_u8_flag, sizeof(int)));
      const int one = 1;
      PXC_CUDA(cudaMemcpyAsync(h->u8_flag.p, &one, sizeof(int), cudaMemcpyHostToDevice, s));
      build_u8_rows_kernel<<<(unsigned)h->nlive, 128, 0, s>>>(h->vectors.p, h->rank_slot.p, h->nlive, dim,
                                                              h->vec_u8.p, h->u8_flag.p);
      PXC_CUDA(cudaGetLastError());
      PXC_CUDA(cudaMemcpyAsync(h->h_u8_flag, h->u8_flag.p, sizeof(int), cudaMemcpyDeviceToHost, s));
      PXC_CUDA(cudaStreamSynchronize(s));
      ctx->launches += 1;
      if (*h->h_u8_flag) h->u8_state = 1;
    }
  }
  // K4: coarse
  const uint32_t P = nprobe;
  const uint32_t batch = 16384;
  const uint32_t cpad = (nlist + 63) / 64 * 64;  // distance-matrix row stride (whole 64-column tiles)
  const uint32_t nbmax = std::min(nq, batch);
  h->probes.reserve((size_t)nbmax * nprobe);
  h->coarse_d.reserve((size_t)nbmax * cpad);
  h->coarse_l.reserve((size_t)nbmax * P);
  h->coarse_len.reserve(nbmax);
  h->coarse_zero.reserve(nbmax);
  PXC_CUDA(cudaMemsetAsync(h->coarse_zero.p, 0, (size_t)nbmax * 4, s));
  // candidate buffer: the shortlist, two chunks of room and the final sort's
  // power of two (at least 4096 entries)
  const uint32_t cb = std::max<uint32_t>(4096, (shortlist + 2 * CHUNK + 1023) / 1024 * 1024);
  const size_t smem_s = (size_t)cb * 8 + ((size_t)h->m * 256 + 2 * dim) * 4 + (2 * h->m + 1) * 4;
  PXC_CUDA(cudaFuncSetAttribute(scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_s));
  if (ctx->profiling) {
    if (!h->ev_begin) PXC_CUDA(cudaEventCreate(&h->ev_begin));
    if (!h->ev_end) PXC_CUDA(cudaEventCreate(&h->ev_end));
  }
  h->timed = false;
  h->scanned.reserve(1);
  PXC_CUDA(cudaMemsetAsync(h->scanned.p, 0, sizeof(unsigned long long), s));
  for (uint32_t q0 = 0; q0 < nq; q0 += batch) {
    const uint32_t nb = std::min(batch, nq - q0);
    const float* qb = d_q + (size_t)q0 * dim;
    dist_chunk_kernel<PXC_EUCLIDEAN><<<dim3(cpad / 64, (nb + 31) / 32), 256, 0, s>>>(
        qb, nb, h->centroids.p, nlist, dim, 0, cpad, nullptr, nullptr, h->coarse_d.p);
    // (an empty input list: coarse_zero holds zero lengths, so coarse_l is not read before it is written)
    select_chunk_kernel<<<nb, SEL_THREADS, 0, s>>>(h->coarse_l.p, h->coarse_zero.p, h->coarse_l.p, h->coarse_len.p,
                                                   h->coarse_d.p, cpad, 0, nlist, P, 0);
    probes_from_lists_kernel<<<nb, 128, 0, s>>>(h->coarse_l.p, h->coarse_len.p, P, nprobe, h->probes.p);
    ScanParams sp{};
    sp.queries = qb;
    sp.probes = h->probes.p;
    sp.centroids = h->centroids.p;
    sp.codebooks = h->codebooks.p;
    sp.woff = h->woff.p;
    sp.list_off = h->list_off.p;
    sp.list_slot = h->list_slot.p;
    sp.list_codes = h->list_codes.p;
    sp.list_rank = h->list_rank.p;
    sp.scanned = h->scanned.p;
    sp.rank_slot = h->rank_slot.p;
    sp.ids = h->ids.p;
    sp.vectors = h->have_vectors ? h->vectors.p : nullptr;
    sp.vec_u8 = (h->have_vectors && h->u8_state == 1) ? h->vec_u8.p : nullptr;
    sp.bitmap = d_bitmap;
    sp.out_ids = d_ids + (size_t)q0 * k;
    sp.out_dist = d_dist + (size_t)q0 * k;
    sp.out_len = d_len + q0;
    sp.nq = nb;
    sp.dim = dim;
    sp.m = h->m;
    sp.nprobe = nprobe;
    sp.k = k;
    sp.shortlist = shortlist;
    sp.cb = cb;
    sp.metric = h->metric;
    sp.rerank = rerank > 0;
    const bool time_it = ctx->profiling && q0 == 0 && nb == nq;  // one batch: time its scan
    if (time_it) PXC_CUDA(cudaEventRecord(h->ev_begin, s));
    scan_kernel<<<nb, SCAN_THREADS, smem_s, s>>>(sp);
    if (time_it) {
      PXC_CUDA(cudaEventRecord(h->ev_end, s));
      h->timed = true;
    }
    PXC_CUDA(cudaGetLastError());
    ctx->launches += 4;
  }
}

// encode_all (ivfpq.rs:828-865) on the device: list_of = nearest centroid in
// squared_euclidean's order, codes = PQ code of the residual, lists rebuilt
// in ascending slot order.
// ProductQuantizer::train's per-subspace loop (product.rs:242-284) on n dense
// device rows of `dim` floats: one ChaCha8 stream seeded once and advanced
// across subspaces, kmeans(projection, width, 256, max_iter, rng) per
// subspace, each codebook padded to 256 entries by repeating its last
// centroid, inertia and iterations summed in subspace order. The caller holds
// ctx->mu (k-means uses the context's workspace).
void pq_train(pxc_ctx* ctx, const float* d_x, uint64_t n, uint32_t dim, const std::vector<uint32_t>& widths,
              const std::vector<uint32_t>& offsets, uint32_t max_iter, uint64_t seed, float* d_books,
              double* inertia, uint64_t* iterations, cudaStream_t s) {
  ChaCha8 prng(seed);
  DBuf<float> proj, book;
  double total = 0.0;
  uint64_t its = 0;
  for (uint32_t sub = 0; sub < (uint32_t)widths.size(); ++sub) {
    const uint32_t w = widths[sub], o = offsets[sub];
    const uint32_t ldw = (w + 3) & ~3u;
    proj.reserve(n * ldw);
    gather_cols_kernel<<<(unsigned)((n * w + 255) / 256), 256, 0, s>>>(d_x, dim, n, o, w, ldw, proj.p);
    book.reserve((size_t)256 * w);
    km::Result r = km::kmeans_impl(ctx, proj.p, ldw, n, w, 256, max_iter, nullptr, &prng, book.p, nullptr, s);
    total += r.inertia;
    its += r.iterations;
    float* dst = d_books + (size_t)256 * o;
    PXC_CUDA(cudaMemcpyAsync(dst, book.p, (size_t)r.k * w * 4, cudaMemcpyDeviceToDevice, s));
    for (uint32_t c = r.k; c < 256; ++c)
      PXC_CUDA(cudaMemcpyAsync(dst + (size_t)c * w, book.p + (size_t)(r.k - 1) * w, w * 4, cudaMemcpyDeviceToDevice,
                               s));
    ctx->launches += 1;
  }
  PXC_CUDA(cudaStreamSynchronize(s));
  *inertia = total;
  *iterations = its;
}

// The (widths, offsets) table of a quantizer as the device kernels read it:
// woff[s] = width, woff[m + s] = offset.
void upload_layout(uint32_t dim, uint32_t m, std::vector<uint32_t>& w, std::vector<uint32_t>& o, DBuf<uint32_t>& woff,
                   cudaStream_t s) {
  layout(dim, m, w, o);
  std::vector<uint32_t> host(2 * m);
  for (uint32_t i = 0; i < m; ++i) {
    host[i] = w[i];
    host[m + i] = o[i];
  }
  woff.reserve(2 * m);
  PXC_CUDA(cudaMemcpyAsync(woff.p, host.data(), 2 * m * 4, cudaMemcpyHostToDevice, s));
}

// Validation shared by the ProductQuantizer entry points (product.rs:199-213).
void check_pq_shape(uint32_t dim, uint32_t m) {
  PXC_CONFIG(dim >= 1 && dim <= MAX_DIM, "dim", dim, "the device quantizer supports 1 <= dim <= 1024");
  PXC_CONFIG(m >= 1 && m <= dim, "subspaces", m, "must be between 1 and the space dimension");
}

// Throws NonFinite{index within its vector} for the first non-finite element.
void check_finite(const float* d_x, uint64_t n, uint32_t dim, cudaStream_t s) {
  if (n == 0) return;
  DBuf<unsigned long long> first;
  first.reserve(1);
  PXC_CUDA(cudaMemsetAsync(first.p, 0xFF, 8, s));
  first_nonfinite_kernel<<<1184, 256, 0, s>>>(d_x, n * dim, first.p);
  PXC_CUDA(cudaGetLastError());
  unsigned long long h = 0;
  PXC_CUDA(cudaMemcpyAsync(&h, first.p, 8, cudaMemcpyDeviceToHost, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  if (h != ~0ull)
    throw make_failure(PXC_NON_FINITE, h % dim, 0, "training", "component %llu of vector %llu is not finite",
                       h % dim, h / dim);
}

void encode_all(pxc_ivfpq* h, cudaStream_t s) {
  pxc_ctx* ctx = h->ctx;
  const uint64_t n = h->nslots;
  const uint32_t dim = h->dim, m = h->m;
  PXC_CONFIG(h->have_parts, "codebooks", 0, "encode needs trained parts");
  PXC_CONFIG(h->have_vectors, "retain_vectors", 0, "encoding needs the full-precision vectors");
  h->list_of.reserve(std::max<uint64_t>(1, n));
  h->codes.reserve(std::max<uint64_t>(16, n * m));
  if (n) {
    km::nearest_rows(ctx, h->vectors.p, dim, n, dim, h->centroids.p, h->nlist, true, h->list_of.p, nullptr, s);
    mask_dead_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(h->list_of.p, h->live.p, n);
    uint32_t wmax = *std::max_element(h->widths.begin(), h->widths.end());
    const size_t smem = ((size_t)256 * wmax + 128 * (wmax + 1)) * 4;
    PXC_CONFIG(smem <= 200 * 1024, "subspaces", m, "subspace too wide for the device encoder");
    PXC_CUDA(cudaFuncSetAttribute(pq_encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    pq_encode_kernel<<<dim3((unsigned)((n + 127) / 128), m), 128, smem, s>>>(
        h->vectors.p, dim, n, h->list_of.p, h->centroids.p, dim, h->codebooks.p, h->woff.p, m, h->codes.p);
    ctx->launches += 2;
  }
  build_lists_device(h, h->list_of.p, s);
}

void build_lists_device(pxc_ivfpq* h, const uint32_t* d_keys, cudaStream_t s) {
  pxc_ctx* ctx = h->ctx;
  const uint64_t n = h->nslots;
  const uint32_t m = h->m;
  // stable sort of slots by list (unassigned last), boundaries, codes in list order
  DBuf<uint32_t> slots, keys_out;
  DBuf<unsigned char> tmp;
  slots.reserve(std::max<uint64_t>(1, n));
  keys_out.reserve(std::max<uint64_t>(1, n));
  h->list_slot.reserve(std::max<uint64_t>(1, n));
  h->list_off.reserve(h->nlist + 1);
  h->list_codes.reserve(std::max<uint64_t>(16, n * m));
  if (n) {
    iota_u32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(slots.p, n);
    size_t tb = 0;
    PXC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tb, d_keys, keys_out.p, slots.p, h->list_slot.p, (int)n, 0, 32,
                                             s));
    tmp.reserve(tb);
    PXC_CUDA(cub::DeviceRadixSort::SortPairs(tmp.p, tb, d_keys, keys_out.p, slots.p, h->list_slot.p, (int)n, 0, 32, s));
    list_bounds_kernel<<<(h->nlist + 256) / 256, 256, 0, s>>>(keys_out.p, n, h->nlist, h->list_off.p);
    gather_codes_kernel<<<(unsigned)((n * m + 255) / 256), 256, 0, s>>>(h->codes.p, m, h->list_slot.p, n,
                                                                       h->list_codes.p);
    h->list_rank.reserve(n);
    list_rank_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(h->list_slot.p, h->slot_rank.p, n, h->list_rank.p);
    ctx->launches += 5;
  } else {
    PXC_CUDA(cudaMemsetAsync(h->list_off.p, 0, (h->nlist + 1) * 4, s));
  }
  PXC_CUDA(cudaGetLastError());
  PXC_CUDA(cudaStreamSynchronize(s));
  h->have_lists = true;
}

void rank_ids_device(pxc_ivfpq* h, const uint32_t* d_live_slots, const uint64_t* d_live_ids, uint64_t nlive,
                     uint32_t* d_dup, cudaStream_t s) {
  const uint64_t n = h->nslots;
  PXC_CONFIG(nlive < (1ull << 31), "nslots", nlive, "the device id ranking sorts fewer than 2^31 live slots");
  h->slot_rank.reserve(std::max<uint64_t>(1, n));
  h->rank_slot.reserve(std::max<uint64_t>(1, nlive));
  if (n) PXC_CUDA(cudaMemsetAsync(h->slot_rank.p, 0xFF, n * 4, s));
  h->nlive = nlive;
  if (!nlive) return;
  DBuf<uint64_t> ids_out;
  DBuf<unsigned char> tmp;
  ids_out.reserve(nlive);
  size_t tb = 0;
  PXC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tb, d_live_ids, ids_out.p, d_live_slots, h->rank_slot.p,
                                           (int)nlive, 0, 64, s));
  tmp.reserve(tb);
  PXC_CUDA(cub::DeviceRadixSort::SortPairs(tmp.p, tb, d_live_ids, ids_out.p, d_live_slots, h->rank_slot.p, (int)nlive,
                                           0, 64, s));
  rank_ids_kernel<<<(unsigned)((nlive + 255) / 256), 256, 0, s>>>(ids_out.p, h->rank_slot.p, nlive, h->slot_rank.p,
                                                                  d_dup);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 3;
  PXC_CUDA(cudaStreamSynchronize(s));  // the sort's scratch is freed on return
}

// The slot store (pxc_ivfpq_set_store / _device): the vectors (host, staged,
// or device) go to HBM and are checked there for non-finite components; the
// VectorId ranks of the live slots are a radix sort on the device, which also
// finds a VectorId live twice. Clears the lists.
void set_store(pxc_ivfpq* h, const float* vectors, bool on_device, const uint64_t* ids, const uint8_t* live,
               uint64_t nslots) {
  PXC_CONFIG(nslots < 0xFFFFFFFFull, "nslots", nslots, "the device IVF-PQ supports fewer than 2^32 slots");
  std::lock_guard<std::mutex> lock(h->mu);
  pxc_ctx* ctx = h->ctx;
  DeviceGuard g(ctx->device);
  cudaStream_t s = ctx->stream;
  handoff_drain(h);
  h->nslots = nslots;
  h->h_ids.resize(nslots);
  h->h_live.assign(nslots, 1);
  std::vector<uint32_t> live_slots;
  std::vector<uint64_t> live_ids;
  live_slots.reserve(nslots);
  live_ids.reserve(nslots);
  for (uint64_t i = 0; i < nslots; ++i) {
    h->h_ids[i] = ids ? ids[i] : i;
    if (live) h->h_live[i] = live[i] ? 1 : 0;
    if (h->h_live[i]) {
      live_slots.push_back((uint32_t)i);
      live_ids.push_back(h->h_ids[i]);
    }
  }
  const uint64_t nlive = live_slots.size();
  DBuf<uint32_t> d_slots, flags;
  DBuf<uint64_t> d_ids;
  DBuf<unsigned long long> first;
  flags.reserve(1);
  first.reserve(1);
  PXC_CUDA(cudaMemsetAsync(flags.p, 0xFF, 4, s));
  PXC_CUDA(cudaMemsetAsync(first.p, 0xFF, 8, s));
  h->have_vectors = false;
  if (vectors && nslots) {
    h->vectors.reserve(nslots * h->dim);
    if (on_device)
      PXC_CUDA(cudaMemcpyAsync(h->vectors.p, vectors, nslots * h->dim * 4, cudaMemcpyDeviceToDevice, s));
    else
      hostcopy::to_device(ctx, h->vectors.p, vectors, nslots * h->dim * 4, s);
    first_nonfinite_kernel<<<1184, 256, 0, s>>>(h->vectors.p, nslots * h->dim, first.p);
    PXC_CUDA(cudaGetLastError());
    ctx->launches += 1;
  }
  h->ids.reserve(std::max<uint64_t>(1, nslots));
  h->live.reserve(std::max<uint64_t>(1, nslots));
  d_slots.reserve(std::max<uint64_t>(1, nlive));
  d_ids.reserve(std::max<uint64_t>(1, nlive));
  hostcopy::to_device(ctx, h->ids.p, h->h_ids.data(), nslots * 8, s);
  hostcopy::to_device(ctx, h->live.p, h->h_live.data(), nslots, s);
  hostcopy::to_device(ctx, d_slots.p, live_slots.data(), nlive * 4, s);
  hostcopy::to_device(ctx, d_ids.p, live_ids.data(), nlive * 8, s);
  rank_ids_device(h, d_slots.p, d_ids.p, nlive, flags.p, s);  // returns synchronised
  unsigned long long bad = 0;
  uint32_t dup = 0;
  PXC_CUDA(cudaMemcpy(&bad, first.p, 8, cudaMemcpyDeviceToHost));
  PXC_CUDA(cudaMemcpy(&dup, flags.p, 4, cudaMemcpyDeviceToHost));
  h->have_lists = false;
  h->u8_state = 0;
  if (bad != ~0ull) {
    h->nslots = 0;
    h->nlive = 0;
    throw make_failure(PXC_NON_FINITE, bad, 0, "vectors", "vector component %llu is not finite", bad);
  }
  if (dup != 0xFFFFFFFFu) {
    h->nslots = 0;
    h->nlive = 0;
    throw make_failure(PXC_DUPLICATE_ID, h->h_ids[dup], 0, "ids", "VectorId %llu is live twice",
                       (unsigned long long)h->h_ids[dup]);
  }
  h->have_vectors = vectors != nullptr && nslots > 0;
}

}  // namespace ivf
}  // namespace pxc

using namespace pxc;

extern "C" {

pxc_status pxc_ivfpq_create(pxc_ctx* ctx, uint32_t dim, int32_t metric, uint32_t nlist, uint32_t m,
                            pxc_ivfpq** out, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(out != nullptr, "out", 0, "output handle pointer is null");
    PXC_CONFIG(dim >= 1 && dim <= ivf::MAX_DIM, "dim", dim, "the device IVF-PQ supports 1 <= dim <= 1024");
    PXC_CONFIG(metric == PXC_EUCLIDEAN || metric == PXC_COSINE, "metric", metric,
               "the device IVF-PQ supports euclidean and cosine");
    PXC_CONFIG(nlist >= 1, "nlist", nlist, "must be at least 1");
    PXC_CONFIG(m >= 1 && m <= dim, "subspaces", m, "must be between 1 and the space dimension");
    PXC_CONFIG(m <= ivf::MAX_M, "subspaces", m, "the device IVF-PQ supports at most 64 subspaces");
    DeviceGuard g(ctx->device);
    auto* h = new pxc_ivfpq();
    h->ctx = ctx;
    h->dim = dim;
    h->metric = metric;
    h->nlist = nlist;
    h->m = m;
    ivf::layout(dim, m, h->widths, h->offsets);
    std::vector<uint32_t> wo(h->widths);
    wo.insert(wo.end(), h->offsets.begin(), h->offsets.end());
    try {
      h->woff.reserve(wo.size());
      PXC_CUDA(cudaMemcpy(h->woff.p, wo.data(), wo.size() * 4, cudaMemcpyHostToDevice));
    } catch (...) {
      delete h;
      throw;
    }
    *out = h;
  });
}

void pxc_ivfpq_destroy(pxc_ivfpq* h) {
  if (!h) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(h->ctx->device);
  delete h;
  if (prev >= 0) cudaSetDevice(prev);
}

pxc_status pxc_ivfpq_set_parts(pxc_ivfpq* h, const float* centroids, const float* codebooks, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr && centroids != nullptr && codebooks != nullptr, "parts", 0, "null argument");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = h->ctx->stream;
    ivf::handoff_drain(h);
    h->centroids.reserve((size_t)h->nlist * h->dim);
    h->codebooks.reserve((size_t)256 * h->dim);
    PXC_CUDA(cudaMemcpyAsync(h->centroids.p, centroids, (size_t)h->nlist * h->dim * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(h->codebooks.p, codebooks, (size_t)256 * h->dim * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    h->have_parts = true;
  });
}

pxc_status pxc_ivfpq_set_store(pxc_ivfpq* h, const float* vectors, const uint64_t* ids, const uint8_t* live,
                               uint64_t nslots, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    ivf::set_store(h, vectors, false, ids, live, nslots);
  });
}

pxc_status pxc_ivfpq_set_store_device(pxc_ivfpq* h, const float* d_vectors, const uint64_t* ids,
                                      const uint8_t* live, uint64_t nslots, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    ivf::set_store(h, d_vectors, true, ids, live, nslots);
  });
}

uint64_t pxc_ivfpq_last_scanned(pxc_ivfpq* h) {
  if (!h || !h->scanned.p) return 0;
  unsigned long long v = 0;
  if (cudaMemcpy(&v, h->scanned.p, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return 0;
  return v;
}

float pxc_ivfpq_last_scan_ms(pxc_ivfpq* h) {
  if (!h || !h->timed) return -1.0f;
  float ms = -1.0f;
  if (cudaEventSynchronize(h->ev_end) != cudaSuccess) return -1.0f;
  if (cudaEventElapsedTime(&ms, h->ev_begin, h->ev_end) != cudaSuccess) return -1.0f;
  return ms;
}

pxc_status pxc_ivfpq_set_codes(pxc_ivfpq* h, const uint32_t* list_of, const uint8_t* codes, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr && (h->nslots == 0 || (list_of && codes)), "codes", 0, "null argument");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    ivf::handoff_drain(h);
    std::vector<uint32_t> lo(list_of, list_of + h->nslots);
    ivf::build_lists(h, lo, codes, h->ctx->stream);
    h->list_of.reserve(std::max<uint64_t>(1, h->nslots));
    h->codes.reserve(std::max<uint64_t>(16, h->nslots * h->m));
    if (h->nslots) {
      PXC_CUDA(cudaMemcpy(h->list_of.p, list_of, h->nslots * 4, cudaMemcpyHostToDevice));
      PXC_CUDA(cudaMemcpy(h->codes.p, codes, h->nslots * h->m, cudaMemcpyHostToDevice));
    }
  });
}

pxc_status pxc_ivfpq_encode_all(pxc_ivfpq* h, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    std::lock_guard<std::mutex> lock(h->mu);
    std::lock_guard<std::mutex> ctx_lock(h->ctx->mu);  // nearest centroid uses the context's workspace
    DeviceGuard g(h->ctx->device);
    ivf::handoff_drain(h);
    ivf::encode_all(h, h->ctx->stream);
  });
}

pxc_status pxc_ivfpq_train(pxc_ivfpq* h, uint64_t training_sample, uint32_t max_iterations, uint64_t seed,
                           pxc_ivfpq_report* report, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    std::lock_guard<std::mutex> lock(h->mu);
    std::lock_guard<std::mutex> ctx_lock(h->ctx->mu);  // k-means uses the context's workspace
    DeviceGuard g(h->ctx->device);
    ivf::handoff_drain(h);
    pxc_ctx* ctx = h->ctx;
    cudaStream_t s = ctx->stream;
    const uint32_t dim = h->dim, m = h->m;
    // ivfpq.rs:736-757
    PXC_CONFIG(h->have_vectors || h->nlive == 0, "retain_vectors", 0,
               "training needs the full-precision vectors, which were dropped");
    std::vector<uint32_t> live;
    for (uint64_t i = 0; i < h->nslots; ++i)
      if (h->h_live[i]) live.push_back((uint32_t)i);
    PXC_CONFIG(!live.empty(), "len", 0, "an empty index has nothing to fit centroids to");
    PXC_CONFIG(max_iterations >= 1, "max_iterations", max_iterations, "must be at least 1");
    // the stride sample (ivfpq.rs:762-768): every stride-th live slot
    const uint64_t stride = std::max<uint64_t>(1, (live.size() + training_sample - 1) / std::max<uint64_t>(1, training_sample));
    std::vector<uint32_t> pick;
    for (uint64_t i = 0; i < live.size(); i += stride) pick.push_back(live[i]);
    const uint64_t ns = pick.size();
    DBuf<uint32_t> rows;
    DBuf<float> sample, residuals, cent, books;
    rows.reserve(ns);
    sample.reserve(ns * dim);
    PXC_CUDA(cudaMemcpyAsync(rows.p, pick.data(), ns * 4, cudaMemcpyHostToDevice, s));
    ivf::gather_rows_kernel<<<(unsigned)((ns * dim + 255) / 256), 256, 0, s>>>(h->vectors.p, dim, rows.p, ns, sample.p);
    // coarse k-means (ivfpq.rs:770-777), ChaCha8 seeded once
    ChaCha8 rng(seed);
    const uint32_t produced = (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(h->nlist, ns));
    cent.reserve((size_t)produced * dim);
    km::Result coarse = km::kmeans_impl(ctx, sample.p, dim, ns, dim, h->nlist, max_iterations, nullptr, &rng, cent.p,
                                        nullptr, s);
    // residuals of the sample to their nearest centroid (8-lane order)
    DBuf<uint32_t> near;
    near.reserve(ns);
    km::nearest_rows(ctx, sample.p, dim, ns, dim, cent.p, produced, true, near.p, nullptr, s);
    residuals.reserve(ns * dim);
    ivf::residual_kernel<<<(unsigned)((ns * dim + 255) / 256), 256, 0, s>>>(sample.p, dim, ns, dim, near.p, cent.p,
                                                                         residuals.p);
    // ProductQuantizer::train (product.rs:198-296) on the residuals, with a
    // fresh ChaCha8 stream of the same seed (ivfpq.rs:794-800)
    books.reserve((size_t)256 * dim);
    double residual_inertia = 0.0;
    uint64_t pq_iterations = 0;
    ivf::pq_train(ctx, residuals.p, ns, dim, h->widths, h->offsets, max_iterations, seed, books.p, &residual_inertia,
                  &pq_iterations, s);
    // install the parts (the list count is what k-means produced) and encode
    h->nlist = produced;
    h->centroids.reserve((size_t)produced * dim);
    h->codebooks.reserve((size_t)256 * dim);
    PXC_CUDA(cudaMemcpyAsync(h->centroids.p, cent.p, (size_t)produced * dim * 4, cudaMemcpyDeviceToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(h->codebooks.p, books.p, (size_t)256 * dim * 4, cudaMemcpyDeviceToDevice, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    h->have_parts = true;
    ivf::encode_all(h, s);
    if (report) {
      std::vector<uint32_t> off(produced + 1);
      PXC_CUDA(cudaMemcpy(off.data(), h->list_off.p, (produced + 1) * 4, cudaMemcpyDeviceToHost));
      uint64_t populated = 0, largest = 0;
      for (uint32_t l = 0; l < produced; ++l) {
        const uint64_t len = off[l + 1] - off[l];
        populated += len > 0;
        largest = std::max(largest, len);
      }
      std::memset(report, 0, sizeof(*report));
      report->sampled = ns;
      report->coarse_inertia = coarse.inertia;
      report->coarse_iterations = coarse.iterations;
      report->residual_inertia = residual_inertia;
      report->populated_lists = populated;
      report->largest_list = largest;
      report->produced = produced;
      report->pq_iterations = pq_iterations;
    }
  });
}

pxc_status pxc_ivfpq_get_parts(pxc_ivfpq* h, float* centroids, float* codebooks, uint32_t* list_of, uint8_t* codes,
                               uint32_t* out_nlist, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = h->ctx->stream;
    if (out_nlist) *out_nlist = h->nlist;
    if (centroids && h->have_parts)
      PXC_CUDA(cudaMemcpyAsync(centroids, h->centroids.p, (size_t)h->nlist * h->dim * 4, cudaMemcpyDeviceToHost, s));
    if (codebooks && h->have_parts)
      PXC_CUDA(cudaMemcpyAsync(codebooks, h->codebooks.p, (size_t)256 * h->dim * 4, cudaMemcpyDeviceToHost, s));
    if (list_of && h->nslots && h->list_of.p)
      PXC_CUDA(cudaMemcpyAsync(list_of, h->list_of.p, h->nslots * 4, cudaMemcpyDeviceToHost, s));
    if (codes && h->nslots && h->codes.p)
      PXC_CUDA(cudaMemcpyAsync(codes, h->codes.p, h->nslots * h->m, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
  });
}

pxc_status pxc_ivfpq_search_device(pxc_ivfpq* h, const float* d_queries, uint32_t nq, uint32_t k, uint32_t nprobe,
                                   uint32_t rerank, const uint64_t* d_bitmap, uint64_t* d_out_ids,
                                   float* d_out_dist, uint32_t* d_out_len, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    PXC_CONFIG(k <= PXC_MAX_K, "k", k, "k exceeds the maximum");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->ctx->stream;
    ivf::handoff_wait(h, s);
    ivf::search_device(h, d_queries, nq, k, nprobe, rerank, d_bitmap, d_out_ids, d_out_dist, d_out_len, s);
    ivf::handoff_done(h, s);
  });
}

pxc_status pxc_ivfpq_search_sharded(pxc_ivfpq* h, const float* d_queries, uint32_t nq, uint32_t k, uint32_t nprobe,
                                    uint32_t rerank, const uint64_t* d_bitmap, uint64_t* d_out_ids, float* d_out_dist,
                                    uint32_t* d_out_len, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    PXC_CONFIG(k <= PXC_MAX_K, "k", k, "k exceeds the maximum");
    pxc_ctx* ctx = h->ctx;
    PXC_CONFIG((uint64_t)ctx->nranks * k <= 8192, "nranks*k", (uint64_t)ctx->nranks * k,
               "the merge holds at most 8192 candidates per query");
    if (nq == 0) return;
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    std::lock_guard<std::mutex> comm_lock(ctx->comm_mu);
    unsigned char* send = exchange_send_buffer(ctx, exchange_segment_bytes(nq, k));
    const size_t n = (size_t)nq * k;
    ivf::handoff_wait(h, s);
    ivf::search_device(h, d_queries, nq, k, nprobe, rerank, d_bitmap, reinterpret_cast<uint64_t*>(send),
                       reinterpret_cast<float*>(send + n * 8), reinterpret_cast<uint32_t*>(send + n * 12), s);
    exchange_and_merge(ctx, send, nq, k, k, d_out_ids, d_out_dist, d_out_len, s);
    ivf::handoff_done(h, s);
  });
}

static pxc_status ivfpq_search_host(pxc_ivfpq* h, const float* queries, uint32_t nq, uint32_t k, uint32_t nprobe,
                                    uint32_t rerank, const uint64_t* bitmap, pxc_columns* cols,
                                    const pxc_condition* conds, uint32_t ncond, const pxc_operand* operands,
                                    uint32_t noperands, uint64_t* out_ids, float* out_dist, uint32_t* out_len,
                                    pxc_error* err);

pxc_status pxc_ivfpq_search(pxc_ivfpq* h, const float* queries, uint32_t nq, uint32_t k, uint32_t nprobe,
                            uint32_t rerank, const uint64_t* bitmap, uint64_t* out_ids, float* out_dist,
                            uint32_t* out_len, pxc_error* err) {
  return ivfpq_search_host(h, queries, nq, k, nprobe, rerank, bitmap, nullptr, nullptr, 0, nullptr, 0, out_ids,
                           out_dist, out_len, err);
}

pxc_status pxc_ivfpq_search_where(pxc_ivfpq* h, pxc_columns* cols, const pxc_condition* conds, uint32_t ncond,
                                  const pxc_operand* operands, uint32_t noperands, const float* queries, uint32_t nq,
                                  uint32_t k, uint32_t nprobe, uint32_t rerank, uint64_t* out_ids, float* out_dist,
                                  uint32_t* out_len, pxc_error* err) {
  if (cols == nullptr) {
    return report(make_failure(PXC_CONFIGURATION, 0, 0, "columns", "null columns handle"), err);
  }
  return ivfpq_search_host(h, queries, nq, k, nprobe, rerank, nullptr, cols, conds, ncond, operands, noperands,
                           out_ids, out_dist, out_len, err);
}

static pxc_status ivfpq_search_host(pxc_ivfpq* h, const float* queries, uint32_t nq, uint32_t k, uint32_t nprobe,
                                    uint32_t rerank, const uint64_t* bitmap, pxc_columns* cols,
                                    const pxc_condition* conds, uint32_t ncond, const pxc_operand* operands,
                                    uint32_t noperands, uint64_t* out_ids, float* out_dist, uint32_t* out_len,
                                    pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    PXC_CONFIG(k <= PXC_MAX_K, "k", k, "k exceeds the maximum");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = h->ctx->stream;
    if (nq == 0) return;
    for (uint64_t i = 0; i < (uint64_t)nq * h->dim; ++i)
      if (!std::isfinite(queries[i]))
        throw make_failure(PXC_NON_FINITE, i, 0, "queries", "query component %llu is not finite",
                           (unsigned long long)i);
    h->q_buf.reserve((size_t)nq * h->dim);
    h->io_ids.reserve((size_t)nq * std::max<uint32_t>(k, 1));
    h->io_dist.reserve((size_t)nq * std::max<uint32_t>(k, 1));
    h->io_len.reserve(nq);
    ivf::handoff_wait(h, s);
    const uint64_t* db = nullptr;
    if (bitmap || cols) {
      const uint64_t words = (h->nslots + 63) / 64;
      h->bitmap.reserve(std::max<uint64_t>(1, words));
      if (words && bitmap) PXC_CUDA(cudaMemcpyAsync(h->bitmap.p, bitmap, words * 8, cudaMemcpyHostToDevice, s));
      if (words && cols) {  // the conditions evaluated on the device into the bitmap
        pxc_error e{};
        if (pxc_columns_eval(cols, h->nslots, conds, ncond, operands, noperands, h->bitmap.p, s, &e) != PXC_OK)
          throw make_failure((pxc_status)e.code, e.a, e.b, e.parameter, "%s", e.detail);
      }
      db = h->bitmap.p;
    }
    PXC_CUDA(cudaMemcpyAsync(h->q_buf.p, queries, (size_t)nq * h->dim * 4, cudaMemcpyHostToDevice, s));
    ivf::search_device(h, h->q_buf.p, nq, k, nprobe, rerank, db, h->io_ids.p, h->io_dist.p, h->io_len.p, s);
    PXC_CUDA(cudaMemcpyAsync(out_len, h->io_len.p, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
    if (k) {
      PXC_CUDA(cudaMemcpyAsync(out_ids, h->io_ids.p, (size_t)nq * k * 8, cudaMemcpyDeviceToHost, s));
      PXC_CUDA(cudaMemcpyAsync(out_dist, h->io_dist.p, (size_t)nq * k * 4, cudaMemcpyDeviceToHost, s));
    }
    ivf::handoff_done(h, s);
    PXC_CUDA(cudaStreamSynchronize(s));
  });
}

// ---------------------------------------------------------------------------
// ProductQuantizer on its own (crates/proxima-quantize/src/product.rs)
// ---------------------------------------------------------------------------
pxc_status pxc_pq_train_device(pxc_ctx* ctx, const float* d_training, uint64_t n, uint32_t dim, uint32_t m,
                               uint32_t max_iterations, uint64_t seed, float* d_out_codebooks, double* out_inertia,
                               uint64_t* out_iterations, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    ivf::check_pq_shape(dim, m);
    PXC_CONFIG(max_iterations >= 1, "max_iterations", max_iterations, "must be at least 1");
    PXC_CONFIG(n >= 1 && d_training != nullptr, "training", n, "must be a non-empty multiple of the space dimension");
    PXC_CONFIG(n <= 0x7FFFFFFFull, "training", n, "the device quantizer trains on fewer than 2^31 vectors");
    PXC_CONFIG(d_out_codebooks != nullptr, "out_codebooks", 0, "null output buffer");
    std::lock_guard<std::mutex> lock(ctx->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    ivf::check_finite(d_training, n, dim, s);
    std::vector<uint32_t> w, o;
    ivf::layout(dim, m, w, o);
    double inertia = 0.0;
    uint64_t its = 0;
    ivf::pq_train(ctx, d_training, n, dim, w, o, max_iterations, seed, d_out_codebooks, &inertia, &its, s);
    if (out_inertia) *out_inertia = inertia;
    if (out_iterations) *out_iterations = its;
  });
}

pxc_status pxc_pq_train(pxc_ctx* ctx, const float* training, uint64_t n, uint32_t dim, uint32_t m,
                        uint32_t max_iterations, uint64_t seed, float* out_codebooks, double* out_inertia,
                        uint64_t* out_iterations, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    ivf::check_pq_shape(dim, m);
    PXC_CONFIG(max_iterations >= 1, "max_iterations", max_iterations, "must be at least 1");
    PXC_CONFIG(n >= 1 && training != nullptr, "training", n, "must be a non-empty multiple of the space dimension");
    PXC_CONFIG(out_codebooks != nullptr, "out_codebooks", 0, "null output buffer");
    DBuf<float> dx, books;
    {
      DeviceGuard g(ctx->device);
      dx.reserve(n * dim);
      books.reserve((size_t)256 * dim);
      // on the context stream, which the device entry point below also uses
      PXC_CUDA(cudaMemcpyAsync(dx.p, training, n * dim * 4, cudaMemcpyHostToDevice, ctx->stream));
    }
    pxc_error e2{};
    if (pxc_pq_train_device(ctx, dx.p, n, dim, m, max_iterations, seed, books.p, out_inertia, out_iterations, nullptr,
                            &e2) != PXC_OK)
      throw make_failure((pxc_status)e2.code, e2.a, e2.b, e2.parameter, "%s", e2.detail);
    DeviceGuard g(ctx->device);
    PXC_CUDA(cudaMemcpy(out_codebooks, books.p, (size_t)256 * dim * 4, cudaMemcpyDeviceToHost));
  });
}

pxc_status pxc_pq_encode_device(pxc_ctx* ctx, const float* d_codebooks, uint32_t dim, uint32_t m,
                                const float* d_vectors, uint64_t n, uint8_t* d_out_codes, void* stream,
                                pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    ivf::check_pq_shape(dim, m);
    if (n == 0) return;
    PXC_CONFIG(d_codebooks && d_vectors && d_out_codes, "buffers", 0, "null buffer");
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    std::vector<uint32_t> w, o;
    DBuf<uint32_t> woff;
    ivf::upload_layout(dim, m, w, o, woff, s);
    const uint32_t wmax = *std::max_element(w.begin(), w.end());
    const size_t smem = ((size_t)256 * wmax + 128 * (wmax + 1)) * 4;
    PXC_CONFIG(smem <= 200 * 1024, "subspaces", m, "subspace too wide for the device encoder");
    PXC_CUDA(cudaFuncSetAttribute(ivf::pq_encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    for (uint64_t b = 0; b < n; b += (1ull << 30)) {  // grid.x stays below 2^31 / 128 blocks per launch
      const uint64_t nb = std::min<uint64_t>(n - b, 1ull << 30);
      ivf::pq_encode_kernel<<<dim3((unsigned)((nb + 127) / 128), m), 128, smem, s>>>(
          d_vectors + b * dim, dim, nb, nullptr, nullptr, dim, d_codebooks, woff.p, m, d_out_codes + b * m);
      PXC_CUDA(cudaGetLastError());
      ctx->launches += 1;
    }
    PXC_CUDA(cudaStreamSynchronize(s));  // woff is freed on return
  });
}

pxc_status pxc_pq_encode(pxc_ctx* ctx, const float* codebooks, uint32_t dim, uint32_t m, const float* vectors,
                         uint64_t n, uint8_t* out_codes, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    ivf::check_pq_shape(dim, m);
    if (n == 0) return;
    PXC_CONFIG(codebooks && vectors && out_codes, "buffers", 0, "null buffer");
    DeviceGuard g(ctx->device);
    cudaStream_t s = ctx->stream;
    std::lock_guard<std::mutex> lock(ctx->mu);  // the context stream
    DBuf<float> db, dv;
    DBuf<uint8_t> dc;
    db.reserve((size_t)256 * dim);
    dv.reserve(n * dim);
    dc.reserve(n * m);
    PXC_CUDA(cudaMemcpyAsync(db.p, codebooks, (size_t)256 * dim * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(dv.p, vectors, n * dim * 4, cudaMemcpyHostToDevice, s));
    pxc_error e2{};
    if (pxc_pq_encode_device(ctx, db.p, dim, m, dv.p, n, dc.p, s, &e2) != PXC_OK)
      throw make_failure((pxc_status)e2.code, e2.a, e2.b, e2.parameter, "%s", e2.detail);
    PXC_CUDA(cudaMemcpyAsync(out_codes, dc.p, n * m, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
  });
}

pxc_status pxc_pq_decode(pxc_ctx* ctx, const float* codebooks, uint32_t dim, uint32_t m, const uint8_t* codes,
                         uint64_t n, float* out, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    ivf::check_pq_shape(dim, m);
    if (n == 0) return;
    PXC_CONFIG(codebooks && codes && out, "buffers", 0, "null buffer");
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lock(ctx->mu);
    cudaStream_t s = ctx->stream;
    std::vector<uint32_t> w, o;
    DBuf<uint32_t> woff;
    ivf::upload_layout(dim, m, w, o, woff, s);
    DBuf<float> db, dout;
    DBuf<uint8_t> dc;
    db.reserve((size_t)256 * dim);
    dc.reserve(n * m);
    dout.reserve(n * dim);
    PXC_CUDA(cudaMemcpyAsync(db.p, codebooks, (size_t)256 * dim * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(dc.p, codes, n * m, cudaMemcpyHostToDevice, s));
    ivf::pq_decode_kernel<<<(unsigned)((n * m + 255) / 256), 256, 0, s>>>(dc.p, n, dim, m, db.p, woff.p, dout.p);
    PXC_CUDA(cudaGetLastError());
    ctx->launches += 1;
    PXC_CUDA(cudaMemcpyAsync(out, dout.p, n * dim * 4, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
  });
}

pxc_status pxc_pq_tables_device(pxc_ctx* ctx, const float* d_codebooks, uint32_t dim, uint32_t m,
                                const float* d_queries, uint32_t nq, float* d_out_squared, float* d_out_dot,
                                void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    ivf::check_pq_shape(dim, m);
    if (nq == 0) return;
    PXC_CONFIG(d_codebooks && d_queries && d_out_squared && d_out_dot, "buffers", 0, "null buffer");
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    std::vector<uint32_t> w, o;
    DBuf<uint32_t> woff;
    ivf::upload_layout(dim, m, w, o, woff, s);
    ivf::pq_tables_kernel<<<dim3(nq, m), 256, 0, s>>>(d_queries, dim, d_codebooks, woff.p, m, d_out_squared,
                                                      d_out_dot);
    PXC_CUDA(cudaGetLastError());
    ctx->launches += 1;
    PXC_CUDA(cudaStreamSynchronize(s));  // woff is freed on return
  });
}

pxc_status pxc_pq_tables(pxc_ctx* ctx, const float* codebooks, uint32_t dim, uint32_t m, const float* queries,
                         uint32_t nq, float* out_squared, float* out_dot, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    ivf::check_pq_shape(dim, m);
    if (nq == 0) return;
    PXC_CONFIG(codebooks && queries && out_squared && out_dot, "buffers", 0, "null buffer");
    DeviceGuard g(ctx->device);
    std::lock_guard<std::mutex> lock(ctx->mu);
    cudaStream_t s = ctx->stream;
    DBuf<float> db, dq, dsq, ddot;
    db.reserve((size_t)256 * dim);
    dq.reserve((size_t)nq * dim);
    dsq.reserve((size_t)nq * m * 256);
    ddot.reserve((size_t)nq * m * 256);
    PXC_CUDA(cudaMemcpyAsync(db.p, codebooks, (size_t)256 * dim * 4, cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(dq.p, queries, (size_t)nq * dim * 4, cudaMemcpyHostToDevice, s));
    pxc_error e2{};
    if (pxc_pq_tables_device(ctx, db.p, dim, m, dq.p, nq, dsq.p, ddot.p, s, &e2) != PXC_OK)
      throw make_failure((pxc_status)e2.code, e2.a, e2.b, e2.parameter, "%s", e2.detail);
    PXC_CUDA(cudaMemcpyAsync(out_squared, dsq.p, (size_t)nq * m * 256 * 4, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaMemcpyAsync(out_dot, ddot.p, (size_t)nq * m * 256 * 4, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
  });
}

}  // extern "C"
