// flat.cu — FlatIndex device mirror and exact batched search.
//
// Replaces the scan of FlatIndex::search (crates/proxima-index/src/flat.rs:153-169).
// Two scan kernels produce the same answer:
//   * K1 (flat_tc.cuh): tcgen05 u8 GEMM + fused top-k, used when the metric is
//     euclidean and every live row and query is an integer in [0,255];
//   * K1g (below): fp32 scan in the reference's exact operation order
//     (8 lane accumulators, pairwise reduce, tail, no FMA), used otherwise.
// Both rank candidates by (total_cmp(distance), id): the device mirror keeps
// the live rows in ascending VectorId order ("rank" order), so a rank index
// breaks ties exactly as the id does.
#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_segmented_radix_sort.cuh>
#include <cub/device/device_select.cuh>
#include <thrust/iterator/counting_iterator.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <new>
#include <vector>

#include <cuda_fp16.h>

#include "common.cuh"
#include "flat_tc.cuh"
#include "refdist.cuh"
#include "fp32scan.cuh"
#include "select.cuh"
#include "tmap.cuh"
#include "topk.cuh"

namespace pxc {

// Final ordering of a K1g list (k <= 2048): sort by (key, rank), map rank to id.
__global__ void finalize_small_kernel(const uint64_t* __restrict__ L, const uint32_t* __restrict__ len,
                                      uint32_t k, uint32_t cap, const uint64_t* __restrict__ rank_id,
                                      uint32_t q_base, uint64_t* __restrict__ out_ids,
                                      float* __restrict__ out_dist, uint32_t* __restrict__ out_len) {
  extern __shared__ uint64_t sl[];
  const uint64_t* Lq = L + (size_t)blockIdx.x * k;
  const uint32_t n = len[blockIdx.x];
  for (uint32_t i = threadIdx.x; i < cap; i += blockDim.x) sl[i] = i < n ? Lq[i] : ~0ull;
  __syncthreads();
  block_bitonic_sort_u64(sl, cap);
  const size_t q = q_base + blockIdx.x;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    uint64_t v = sl[i];
    out_ids[q * k + i] = rank_id[static_cast<uint32_t>(v)];
    out_dist[q * k + i] = key_to_float(static_cast<uint32_t>(v >> 32));
  }
  if (threadIdx.x == 0) out_len[q] = n;
}

// Same for already-sorted lists (large k, sorted with the segmented radix sort).
__global__ void finalize_sorted_kernel(const uint64_t* __restrict__ L, const uint32_t* __restrict__ len,
                                       uint32_t k, const uint64_t* __restrict__ rank_id,
                                       uint32_t q_base, uint64_t* __restrict__ out_ids,
                                       float* __restrict__ out_dist, uint32_t* __restrict__ out_len) {
  const uint64_t* Lq = L + (size_t)blockIdx.x * k;
  const uint32_t n = len[blockIdx.x];
  const size_t q = q_base + blockIdx.x;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    uint64_t v = Lq[i];
    out_ids[q * k + i] = rank_id[static_cast<uint32_t>(v)];
    out_dist[q * k + i] = key_to_float(static_cast<uint32_t>(v >> 32));
  }
  if (threadIdx.x == 0) out_len[q] = n;
}

// Unused list tail must not be read as keys by the segmented sort.
__global__ void pad_lists_kernel(uint64_t* L, const uint32_t* len, uint32_t k) {
  uint64_t* Lq = L + (size_t)blockIdx.x * k;
  for (uint32_t i = len[blockIdx.x] + threadIdx.x; i < k; i += blockDim.x) Lq[i] = ~0ull;
}

// ---------------------------------------------------------------------------
// Mirror maintenance
// ---------------------------------------------------------------------------
// Validate a staged range (finite) and classify rows (integers in [0,255]).
__global__ void validate_rows_kernel(const float* __restrict__ rows, uint64_t n, uint32_t dim,
                                     unsigned long long* __restrict__ first_bad,
                                     uint8_t* __restrict__ rowflag) {
  uint64_t r = blockIdx.x;
  if (r >= n) return;
  __shared__ int not_u8;
  if (threadIdx.x == 0) not_u8 = 0;
  __syncthreads();
  for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) {
    float v = rows[r * dim + d];
    if (!isfinite(v)) atomicMin(first_bad, (unsigned long long)(r * dim + d));
    if (!(v >= 0.0f && v <= 255.0f && v == floorf(v))) not_u8 = 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) rowflag[r] = not_u8 ? 0 : 1;
}

__global__ void iota_ids_kernel(uint64_t* ids, uint64_t begin, uint64_t n) {
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) ids[i] = begin + i;
}

__global__ void iota_u32_kernel(uint32_t* v, uint64_t n) {
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) v[i] = static_cast<uint32_t>(i);
}

__global__ void gather_ids_kernel(const uint32_t* slots, const uint64_t* ids, uint64_t* out, uint64_t n) {
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = ids[slots[i]];
}

__global__ void gather_rows_kernel(const uint32_t* __restrict__ rank_slot, const float* __restrict__ rows,
                                   const uint8_t* __restrict__ rowflag, uint32_t dim,
                                   float* __restrict__ out, int* __restrict__ all_u8) {
  uint64_t r = blockIdx.x;
  uint32_t s = rank_slot[r];
  for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) out[r * dim + d] = rows[(uint64_t)s * dim + d];
  if (threadIdx.x == 0 && !rowflag[s]) atomicAnd(all_u8, 0);
}

// u8 operand for K1: row-major [nrank_pad][dp], zero-padded; norms with BIG
// for padding rows.
__global__ void build_u8_operand_kernel(const float* __restrict__ rank_rows, uint64_t nrank,
                                        uint32_t dim, uint32_t dp, uint8_t* __restrict__ op,
                                        int32_t* __restrict__ norms) {
  uint64_t r = blockIdx.x;
  __shared__ int32_t acc;
  if (threadIdx.x == 0) acc = 0;
  __syncthreads();
  int32_t local = 0;
  for (uint32_t d = threadIdx.x; d < dp; d += blockDim.x) {
    uint8_t v = 0;
    if (r < nrank && d < dim) v = static_cast<uint8_t>(rank_rows[r * dim + d]);
    op[r * dp + d] = v;
    local += static_cast<int32_t>(v) * static_cast<int32_t>(v);
  }
  atomicAdd(&acc, local);
  __syncthreads();
  if (threadIdx.x == 0) norms[r] = r < nrank ? acc : flat_tc::BIG;
}

// Filtered K1: one flag per rank (the filter bitmap is over slots).
__global__ void rank_flags_kernel(const uint32_t* __restrict__ rank_slot, uint64_t nrank,
                                  const uint64_t* __restrict__ bitmap, uint8_t* __restrict__ flags) {
  for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < nrank; r += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t slot = rank_slot[r];
    flags[r] = static_cast<uint8_t>((bitmap[slot >> 6] >> (slot & 63)) & 1ull);
  }
}

// Filtered K1 operand: row i (of npad) = u8 row acc[i] (zero past nacc), its
// ||x||^2 (BIG past nacc: never selected) and VectorId. The accepted ranks are
// in ascending rank order, so the compacted index orders as the id does.
__global__ void gather_operand_kernel(const uint8_t* __restrict__ op, const int32_t* __restrict__ norms,
                                      const uint64_t* __restrict__ rank_id, const uint32_t* __restrict__ acc,
                                      uint64_t nacc, uint32_t dp, uint8_t* __restrict__ out_op,
                                      int32_t* __restrict__ out_norm, uint64_t* __restrict__ out_id) {
  const uint64_t i = blockIdx.x;
  const uint4* src = i < nacc ? reinterpret_cast<const uint4*>(op + (uint64_t)acc[i] * dp) : nullptr;
  uint4* dst = reinterpret_cast<uint4*>(out_op + i * dp);
  for (uint32_t w = threadIdx.x; w < dp / 16; w += blockDim.x) dst[w] = src ? __ldg(src + w) : make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    out_norm[i] = i < nacc ? norms[acc[i]] : flat_tc::BIG;
    if (i < nacc) out_id[i] = rank_id[acc[i]];
  }
}

// Queries for K1: u8 tile [nq_pad][dp], ||q||^2, and a flag if any query
// component is not an integer in [0,255] (then K1 does not apply).
__global__ void prep_queries_u8_kernel(const float* __restrict__ Q, uint32_t nq, uint32_t dim,
                                       uint32_t dp, uint8_t* __restrict__ qop,
                                       int32_t* __restrict__ qnorm, int* __restrict__ bad) {
  uint32_t q = blockIdx.x;
  __shared__ int32_t acc;
  if (threadIdx.x == 0) acc = 0;
  __syncthreads();
  int32_t local = 0;
  for (uint32_t d = threadIdx.x; d < dp; d += blockDim.x) {
    uint8_t v = 0;
    if (q < nq && d < dim) {
      float f = Q[(size_t)q * dim + d];
      if (f >= 0.0f && f <= 255.0f && f == floorf(f)) {
        v = static_cast<uint8_t>(f);
      } else {
        atomicExch(bad, 1);
      }
    }
    qop[(size_t)q * dp + d] = v;
    local += static_cast<int32_t>(v) * static_cast<int32_t>(v);
  }
  atomicAdd(&acc, local);
  __syncthreads();
  if (threadIdx.x == 0) qnorm[q] = acc;
}

// Merge of K1's per-split lists: per query, nsplit*KT packed (r, rank) keys,
// sort, drop duplicates (a split may carry entries seeded from an earlier
// split), keep k, distance = r + ||q||^2 (exact integer in f32).
// With counts set (collect mode: per query nsplit unordered segments of KT
// slots, counts [nq][nsplit]) the filled part of every segment is gathered,
// at most cap keys (a query with more overflowed and is answered again).
// Launched with 256 threads per block (one block per query); cap <= 2048, a
// power of two; nsplit <= MERGE_MAX_SPLITS with counts.
constexpr uint32_t MERGE_MAX_SPLITS = 64;
__global__ void __launch_bounds__(256) merge_u8_kernel(const uint64_t* __restrict__ part, uint32_t nsplit, uint32_t KT,
                                uint32_t cap, uint32_t k, const int32_t* __restrict__ qnorm,
                                const uint64_t* __restrict__ rank_id, uint32_t nrank,
                                uint64_t* __restrict__ out_ids, float* __restrict__ out_dist,
                                uint32_t* __restrict__ out_len, const uint32_t* __restrict__ counts) {
  extern __shared__ uint64_t sl[];
  const uint32_t q = blockIdx.x;
  const uint32_t n = nsplit * KT;
  const uint64_t empty_key = static_cast<uint64_t>(static_cast<uint32_t>(flat_tc::BIG) + flat_tc::R_OFFSET) << 32;
  if (counts != nullptr) {
    __shared__ uint32_t seg_off[MERGE_MAX_SPLITS + 1];
    if (threadIdx.x == 0) {
      uint32_t a = 0;
      for (uint32_t sp = 0; sp < nsplit; ++sp) {
        seg_off[sp] = a;
        a += min(counts[(size_t)q * nsplit + sp], KT);
      }
      seg_off[nsplit] = a;
    }
    __syncthreads();
    const uint32_t filled = min(seg_off[nsplit], cap);
    uint32_t sz = 32;  // sort only the filled prefix, rounded up to a power of two (<= cap)
    while (sz < filled) sz <<= 1;
    cap = sz;
    for (uint32_t i = threadIdx.x; i < cap; i += blockDim.x) sl[i] = ~0ull;
    __syncthreads();
    for (uint32_t sp = 0; sp < nsplit; ++sp) {
      const uint32_t b = seg_off[sp], len = seg_off[sp + 1] - b;
      for (uint32_t j = threadIdx.x; j < len && b + j < cap; j += blockDim.x) {
        const uint64_t v = part[(size_t)q * n + (size_t)sp * KT + j];
        sl[b + j] = (v >= empty_key || static_cast<uint32_t>(v) >= nrank) ? ~0ull : v;
      }
    }
  } else {
    for (uint32_t i = threadIdx.x; i < cap; i += blockDim.x) {
      uint64_t v = i < n ? part[(size_t)q * n + i] : ~0ull;
      // empty slots, and (defensively) any rank outside the mirror, never reach the output
      sl[i] = (v >= empty_key || static_cast<uint32_t>(v) >= nrank) ? ~0ull : v;
    }
  }
  __syncthreads();
  block_bitonic_sort_u64(sl, cap);
  // mark duplicates of the previous key, then compact the unique prefix
  __shared__ uint32_t flag[2048];
  for (uint32_t i = threadIdx.x; i < cap; i += blockDim.x)
    flag[i] = (sl[i] != ~0ull && (i == 0 || sl[i] != sl[i - 1])) ? 1u : 0u;
  __syncthreads();
  // Each thread takes a contiguous run of the sorted keys; an exclusive scan of
  // the per-run unique counts gives each run its first output position, so the
  // id lookups of one query's k results are issued in parallel.
  using Scan = cub::BlockScan<uint32_t, 256>;
  __shared__ typename Scan::TempStorage scan_tmp;
  const uint32_t per = (cap + 255) / 256;
  const uint32_t b = threadIdx.x * per;
  const uint32_t e = min(b + per, cap);
  uint32_t cnt = 0;
  for (uint32_t i = b; i < e; ++i) cnt += flag[i];
  uint32_t pos = 0, total = 0;
  Scan(scan_tmp).ExclusiveSum(cnt, pos, total);
  const int32_t qn = qnorm[q];
  for (uint32_t i = b; i < e && pos < k; ++i) {
    if (!flag[i]) continue;
    const uint64_t v = sl[i];
    const int32_t r = static_cast<int32_t>(static_cast<uint32_t>(v >> 32) - flat_tc::R_OFFSET);
    out_ids[(size_t)q * k + pos] = rank_id[static_cast<uint32_t>(v)];
    out_dist[(size_t)q * k + pos] = static_cast<float>(r + qn);
    ++pos;
  }
  if (threadIdx.x == 0) out_len[q] = min(total, k);
}

__global__ void zero_u32_kernel(uint32_t* p, uint64_t n) {
  uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = 0;
}

inline unsigned grid1d(uint64_t n, unsigned block) { return (unsigned)((n + block - 1) / block); }

// K1 keeps at most TC_MAX_K entries per query row; k up to GROUPED_MAX_K runs
// as GROUP_K searches over disjoint rank groups (search_tc_grouped).
constexpr uint32_t TC_MAX_K = 32;
constexpr uint32_t GROUP_K = 32;
constexpr uint32_t GROUPED_MAX_K = 128;

// Exactness of a grouped search, per query. Each group list is that group's
// own top GROUP_K among its rows with r <= T (the shared starting bound, which
// at least k rows meet; T is "none" without the sample pass), so every row
// missing from the union of the lists lies behind the true k-th (r > T) or
// behind the last entry of its group's full list. When every full group list
// ends at or behind the merged k-th entry (by (total_cmp(distance), id)), no
// missing row can be among the first k and the merged list is the exact
// answer. Otherwise (32 or more of the query's top k in one group, or fewer
// than k merged entries while a group list is full) the query is flagged for
// K1g.
__global__ void group_check_kernel(const uint64_t* __restrict__ gids, const float* __restrict__ gdist,
                                   const uint32_t* __restrict__ glen, uint32_t ngroups, uint32_t nq,
                                   const uint64_t* __restrict__ ids, const float* __restrict__ dist,
                                   const uint32_t* __restrict__ len, uint32_t k, uint8_t* __restrict__ redo) {
  const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const bool have_k = len[q] >= k;
  const uint32_t kth_key = have_k ? order_key(dist[(size_t)q * k + k - 1]) : 0u;
  const uint64_t kth_id = have_k ? ids[(size_t)q * k + k - 1] : 0ull;
  uint8_t bad = 0;
  for (uint32_t g = 0; g < ngroups && !bad; ++g) {
    const size_t row = (size_t)g * nq + q;
    if (glen[row] < GROUP_K) continue;  // the whole group is in the union
    if (!have_k) {
      bad = 1;
      break;
    }
    const uint32_t key = order_key(gdist[row * GROUP_K + GROUP_K - 1]);
    const uint64_t id = gids[row * GROUP_K + GROUP_K - 1];
    if (key < kth_key || (key == kth_key && id < kth_id)) bad = 1;
  }
  redo[q] = bad;
}

// Row i of out = query idx[i].
__global__ void gather_queries_kernel(const float* __restrict__ q, const uint32_t* __restrict__ idx,
                                      uint32_t dim, float* __restrict__ out) {
  const size_t src = (size_t)idx[blockIdx.x] * dim;
  const size_t dst = (size_t)blockIdx.x * dim;
  for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) out[dst + d] = q[src + d];
}

// Result row i replaces the result of query idx[i].
__global__ void scatter_results_kernel(const uint64_t* __restrict__ ids, const float* __restrict__ dist,
                                       const uint32_t* __restrict__ len, const uint32_t* __restrict__ idx,
                                       uint32_t k, uint64_t* __restrict__ out_ids, float* __restrict__ out_dist,
                                       uint32_t* __restrict__ out_len) {
  const uint32_t q = idx[blockIdx.x];
  const uint32_t n = len[blockIdx.x];
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    out_ids[(size_t)q * k + i] = ids[(size_t)blockIdx.x * k + i];
    out_dist[(size_t)q * k + i] = dist[(size_t)blockIdx.x * k + i];
  }
  if (threadIdx.x == 0) out_len[q] = n;
}

// ---------------------------------------------------------------------------
// K2: the tensor-core path for non-integer data (euclidean, cosine, inner
// product). A screen on kind::f16 tensor cores (flat_tc.cuh, F16Scan) keeps
// each query's K2_KT best rows by an approximate score d~; the candidates are
// re-scored with the reference's exact f32 distance (8-lane order) and sorted
// by (total_cmp, id); a query's answer is proven exact when every row the
// screen did not keep is provably behind the k-th exact distance:
//   d_ref(x) >= d~(x) - E_s - E_ref >= d~_KT - E_s - E_ref > d_k,
// with E_s a rigorous bound on |d~ - d| (the f16 rounding of both operands,
// the tensor core's f32 accumulation, the centring and the f32 epilogue) and
// E_ref the reference's own rounding. Queries that cannot be proven are
// searched again on K1g. The screen works on rows and queries centred on the
// rows' mean (which shrinks the operands, and with them the bound) and
// scaled by powers of two so that the f16 values use the full range.
// ---------------------------------------------------------------------------
constexpr uint32_t K2_KT = 32;         // candidates the screen keeps per query
constexpr uint32_t K2_MAX_K = 24;      // largest k served (the rest of the list is the proof's margin)
constexpr uint32_t K2_MAX_DIM = 128;   // two 128-byte K blocks of f16
constexpr uint32_t K2_MEAN_CHUNKS = 64;
constexpr uint32_t K2_RANGE_BATCH = 256;  // redo queries per range pass (256 x 32 KiB of collection)

// Partial column sums (f64) of the rank-ordered rows: block (32 columns x 8
// row lanes) per (column group, row chunk); column_mean_kernel folds the
// chunks in order, so the mean does not depend on scheduling.
__global__ void column_partial_kernel(const float* __restrict__ rows, uint64_t n, uint32_t dim,
                                      double* __restrict__ part) {
  const uint32_t col = blockIdx.x * 32 + threadIdx.x;
  const uint64_t per = (n + gridDim.y - 1) / gridDim.y;
  const uint64_t r0 = (uint64_t)blockIdx.y * per, r1 = min(n, r0 + per);
  double acc = 0.0;
  if (col < dim)
    for (uint64_t r = r0 + threadIdx.y; r < r1; r += 8) acc += (double)rows[r * dim + col];
  __shared__ double red[8][33];
  red[threadIdx.y][threadIdx.x] = acc;
  __syncthreads();
  if (threadIdx.y == 0 && col < dim) {
    double t = 0.0;
    for (int i = 0; i < 8; ++i) t += red[i][threadIdx.x];
    part[(size_t)blockIdx.y * dim + col] = t;
  }
}
__global__ void column_mean_kernel(const double* __restrict__ part, uint32_t chunks, uint32_t dim, uint64_t n,
                                   float* __restrict__ mu) {
  const uint32_t col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= dim) return;
  double t = 0.0;
  for (uint32_t c = 0; c < chunks; ++c) t += part[(size_t)c * dim + col];
  mu[col] = (float)(t / (double)n);
}

// Ranges the screen's scale and bound need, over the centred rows:
// [0] max |x'_i|, [1] max ||x'||, [2] max ||x|| (uncentred), [3] max |h_x|,
// each as the bits of a non-negative float rounded up (atomicMax on bits).
__device__ __forceinline__ float round_up_f32(double v) {
  float f = (float)v;
  return ((double)f < v) ? nextafterf(f, INFINITY) : f;
}
__global__ void k2_row_stats_kernel(const float* __restrict__ rows, uint64_t n, uint32_t dim,
                                    const float* __restrict__ mu, int metric, float* __restrict__ h_out,
                                    uint32_t* __restrict__ stats) {
  const uint64_t r = blockIdx.x;
  double c2 = 0.0, u2 = 0.0, mx = 0.0;
  float amax = 0.0f;
  for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) {
    const float x = rows[r * dim + d];
    const float xc = __fsub_rn(x, mu[d]);
    c2 += (double)xc * xc;
    u2 += (double)x * x;
    mx += (double)mu[d] * xc;
    amax = fmaxf(amax, fabsf(xc));
  }
  using Red = cub::BlockReduce<double, 128>;
  __shared__ typename Red::TempStorage t1, t2, t3;
  __shared__ float s_amax;
  if (threadIdx.x == 0) s_amax = 0.0f;
  __syncthreads();
  atomicMax(reinterpret_cast<unsigned*>(&s_amax), __float_as_uint(amax));
  const double C2 = Red(t1).Sum(c2);
  const double U2 = Red(t2).Sum(u2);
  const double MX = Red(t3).Sum(mx);
  __syncthreads();
  if (threadIdx.x == 0) {
    const double h = metric == PXC_EUCLIDEAN ? C2 : -MX;
    h_out[r] = (float)h;
    atomicMax(stats + 0, __float_as_uint(s_amax));
    atomicMax(stats + 1, __float_as_uint(round_up_f32(sqrt(C2))));
    atomicMax(stats + 2, __float_as_uint(round_up_f32(sqrt(U2))));
    atomicMax(stats + 3, __float_as_uint(round_up_f32(fabs(h))));
  }
}

// f16 operand: row r = fl16((x_r - mu) * 2^ax) (rank order; zero padding),
// padding rows' term = F16Scan::big().
__global__ void k2_operand_kernel(const float* __restrict__ rows, uint64_t n, uint32_t dim, uint32_t dp,
                                  const float* __restrict__ mu, int ax, __half* __restrict__ op,
                                  float* __restrict__ h) {
  const uint64_t r = blockIdx.x;
  for (uint32_t d = threadIdx.x; d < dp; d += blockDim.x) {
    float v = 0.0f;
    if (r < n && d < dim) v = ldexpf(__fsub_rn(rows[r * dim + d], mu[d]), ax);
    op[r * dp + d] = __float2half_rn(v);
  }
  if (threadIdx.x == 0 && r >= n) h[r] = flat_tc::F16Scan::big();
}

// Per query: the f16 operand row, the factor c_q, the constant that turns
// the screen's r into d~, and the two error terms of the proof.
struct K2Query {
  float coef;      // c_q
  float cst;       // d~ = r + cst
  double eps;      // E_s: |d~ - d_real| <= eps for every row
  double eref;     // cosine / IP: |d_ref - d_real| <= eref; euclidean: relative factor gamma
  float delta;     // margin of the shared bound over the k-th screened value (> 2 E_s + E_ref)
};
__global__ void k2_prep_queries_kernel(const float* __restrict__ Q, uint32_t nq, uint32_t dim, uint32_t dp,
                                       const float* __restrict__ mu, int metric, int ax, const float* __restrict__ xst,
                                       __half* __restrict__ qop, K2Query* __restrict__ meta) {
  const uint32_t q = blockIdx.x;
  double c2 = 0.0, u2 = 0.0, qm = 0.0;
  float amax = 0.0f;
  if (q < nq) {
    for (uint32_t d = threadIdx.x; d < dim; d += blockDim.x) {
      const float x = Q[(size_t)q * dim + d];
      const float xc = __fsub_rn(x, mu[d]);
      c2 += (double)xc * xc;
      u2 += (double)x * x;
      qm += (double)x * mu[d];
      amax = fmaxf(amax, fabsf(xc));
    }
  }
  using Red = cub::BlockReduce<double, 128>;
  __shared__ typename Red::TempStorage t1, t2, t3;
  __shared__ float s_amax;
  __shared__ int s_aq;
  if (threadIdx.x == 0) s_amax = 0.0f;
  __syncthreads();
  atomicMax(reinterpret_cast<unsigned*>(&s_amax), __float_as_uint(amax));
  const double C2 = Red(t1).Sum(c2);
  const double U2 = Red(t2).Sum(u2);
  const double QM = Red(t3).Sum(qm);
  __syncthreads();
  if (threadIdx.x == 0) s_aq = s_amax > 0.0f ? 14 - ilogbf(s_amax) : 0;
  __syncthreads();
  const int aq = s_aq;
  for (uint32_t d = threadIdx.x; d < dp; d += blockDim.x) {
    float v = 0.0f;
    if (q < nq && d < dim) v = ldexpf(__fsub_rn(Q[(size_t)q * dim + d], mu[d]), aq);
    qop[(size_t)q * dp + d] = __float2half_rn(v);
  }
  if (threadIdx.x != 0) return;
  K2Query m;
  const double k = metric == PXC_EUCLIDEAN ? 2.0 : 1.0;
  m.coef = (float)(-k * ldexp(1.0, -(aq + ax)));
  m.cst = (float)(metric == PXC_EUCLIDEAN ? C2 : (metric == PXC_COSINE ? 1.0 - QM : -QM));
  const double Qn = sqrt(C2) * (1.0 + 1e-12), Qu = sqrt(U2) * (1.0 + 1e-12);
  const double M = xst[1], Mu = xst[2], Hmax = xst[3];
  const double D = (double)dim, u = ldexp(1.0, -11);
  const double A = ldexp(Qn, aq), B = ldexp(M, ax), sub = ldexp(1.0, -25) * sqrt(D);
  const double e_f16 = (2.0 * u + u * u) * A * B + ldexp(1.0, -25) * (1.0 + u) * sqrt(D) * (A + B) +
                       D * ldexp(1.0, -50);
  const double e_acc = D * ldexp(1.0, -23) * (A * (1.0 + u) + sub) * (B * (1.0 + u) + sub);
  const double scale = k * ldexp(1.0, -(aq + ax));
  const double e_dot = (e_f16 + e_acc) * scale;
  const double qmn = k * Qn * M * 1.01;
  const double e_center = metric == PXC_EUCLIDEAN ? ldexp(1.0, -23) * (Qn + M) * (Qn + M) * 1.01
                                                  : ldexp(1.0, -24) * M * (Qu + Qn) * 1.01;
  const double e_round = ldexp(1.0, -22) * (Hmax + qmn + fabs((double)m.cst) + 1.0);
  m.eps = 1.02 * (e_dot + e_center + e_round) + 1e-30;
  const double gamma = (D / 8.0 + 8.0) * ldexp(1.0, -24) * 1.1;
  m.eref = metric == PXC_EUCLIDEAN ? gamma : gamma * Qu * Mu + ldexp(1.0, -24) * (1.0 + Qu * Mu);
  // a query whose factors leave the f32 range cannot be screened; it is proven never
  if (!(isfinite(m.coef) && isfinite(m.cst) && isfinite(m.eps)) || q >= nq) m.eps = INFINITY;
  // A row whose screened value is behind the k-th by more than 2 E_s + E_ref
  // (plus the reference's relative error at that size) is provably behind the
  // k-th exact distance; sharing kth + delta lets the screen drop it.
  const double ref_part = metric == PXC_EUCLIDEAN ? m.eref * (fabs((double)m.cst) + Hmax + qmn) * 2.0 : m.eref;
  m.delta = round_up_f32(1.25 * (2.0 * m.eps + ref_part) + 1e-30);
  meta[q] = m;
}

__global__ void copy_coef_kernel(const K2Query* __restrict__ meta, uint32_t n, float* __restrict__ coef,
                                 float* __restrict__ delta) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    coef[i] = meta[i].coef;
    delta[i] = meta[i].delta;
  }
}

// space.distance on prepared operands (crates/proxima-core/src/space.rs:148-156).
__device__ __forceinline__ float k2_ref_distance(int metric, const float* q, const float* __restrict__ x,
                                                 uint32_t dim) {
  if (metric == PXC_EUCLIDEAN) return l2_unrolled(q, x, dim);
  const float s = dot_unrolled(q, x, dim);
  return metric == PXC_COSINE ? __fsub_rn(1.0f, s) : -s;
}

// Per query: the union of the screen's split lists (sorted, duplicates
// dropped), its first K2_KT entries re-scored exactly and sorted by
// (total_cmp, id), the first k written out, and the proof. 128 threads.
__global__ void __launch_bounds__(128) k2_rerank_kernel(const uint64_t* __restrict__ part, uint32_t nsplit, uint32_t cap,
                                                        const uint32_t* __restrict__ bound,
                                                        const K2Query* __restrict__ meta, const float* __restrict__ Q,
                                                        uint32_t dim, int metric, const float* __restrict__ rank_rows,
                                                        const uint64_t* __restrict__ rank_id, uint32_t nrank, uint32_t k,
                                                        uint64_t* __restrict__ out_ids, float* __restrict__ out_dist,
                                                        uint32_t* __restrict__ out_len, uint8_t* __restrict__ redo,
                                                        float* __restrict__ kth_out) {
  extern __shared__ uint64_t sl[];  // [cap]
  __shared__ uint32_t flag[2048];
  __shared__ uint64_t cand[K2_KT];
  __shared__ uint32_t ncand;
  const uint32_t q = blockIdx.x;
  const uint32_t n = nsplit * K2_KT;
  const uint32_t empty = flat_tc::F16Scan::pack(flat_tc::F16Scan::big());
  for (uint32_t i = threadIdx.x; i < cap; i += blockDim.x) {
    const uint64_t v = i < n ? part[(size_t)q * n + i] : ~0ull;
    sl[i] = (static_cast<uint32_t>(v >> 32) >= empty || static_cast<uint32_t>(v) >= nrank) ? ~0ull : v;
  }
  __syncthreads();
  block_bitonic_sort_u64(sl, cap);
  for (uint32_t i = threadIdx.x; i < cap; i += blockDim.x)
    flag[i] = (sl[i] != ~0ull && (i == 0 || sl[i] != sl[i - 1])) ? 1u : 0u;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t c = 0;
    for (uint32_t i = 0; i < cap && c < K2_KT + 1; ++i) {
      if (!flag[i]) continue;
      if (c < K2_KT) cand[c] = sl[i];
      ++c;
    }
    ncand = c;  // K2_KT + 1 means: more rows were seen than the list keeps
  }
  __syncthreads();
  const uint32_t nc = min(ncand, K2_KT);
  // exact distances of the candidates (one thread each), keyed by (distance, rank)
  __shared__ uint64_t ex[K2_KT];
  const float* qrow = Q + (size_t)q * dim;
  if (threadIdx.x < K2_KT) {
    uint64_t key = ~0ull;
    if (threadIdx.x < nc) {
      const uint32_t rank = static_cast<uint32_t>(cand[threadIdx.x]);
      const float d = k2_ref_distance(metric, qrow, rank_rows + (size_t)rank * dim, dim);
      key = (static_cast<uint64_t>(order_key(d)) << 32) | rank;
    }
    ex[threadIdx.x] = key;
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // warp bitonic sort of the 32 keys
    uint64_t v = ex[threadIdx.x];
    for (uint32_t size = 2; size <= 32; size <<= 1)
      for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
        const uint64_t o = __shfl_xor_sync(0xFFFFFFFFu, v, stride);
        const bool up = (threadIdx.x & size) == 0;
        const bool lower = (threadIdx.x & stride) == 0;
        v = (lower == up) ? (v < o ? v : o) : (v < o ? o : v);
      }
    ex[threadIdx.x] = v;
  }
  __syncthreads();
  const uint32_t take = min(nc, k);
  for (uint32_t i = threadIdx.x; i < take; i += blockDim.x) {
    const uint64_t v = ex[i];
    out_ids[(size_t)q * k + i] = rank_id[static_cast<uint32_t>(v)];
    out_dist[(size_t)q * k + i] = key_to_float(static_cast<uint32_t>(v >> 32));
  }
  if (threadIdx.x == 0) {
    out_len[q] = take;
    // Every row the candidates leave out has r >= T: the shared bound turned
    // it away (r > the final bound), or a full split list did (r >= that
    // list's last entry >= the union's K2_KT-th), or it is behind the union's
    // K2_KT-th entry. T = big: no row was left out.
    using F = flat_tc::F16Scan;
    float T = F::unpack(min(bound[q], F::pack(F::big())));
    if (ncand >= K2_KT) T = fminf(T, F::unpack(static_cast<uint32_t>(cand[K2_KT - 1] >> 32)));
    uint8_t bad = 0;
    if (T < F::big()) {
      const K2Query m = meta[q];
      double lower = (double)T + (double)m.cst - m.eps;
      if (metric == PXC_EUCLIDEAN)
        lower = lower > 0.0 ? lower * (1.0 - m.eref) : lower * (1.0 + m.eref);
      else
        lower -= m.eref;
      const double dk = take ? (double)key_to_float(static_cast<uint32_t>(ex[take - 1] >> 32)) : INFINITY;
      bad = (take < k || !(lower > dk)) ? 1 : 0;
    }
    redo[q] = bad;
    // the candidates' k-th exact distance bounds the true k-th from above
    kth_out[q] = take == k ? key_to_float(static_cast<uint32_t>(ex[take - 1] >> 32)) : INFINITY;
  }
}

// The screen's fallback for the queries it could not prove: every row's
// exact distance, and the rows at or ahead of the candidates' k-th exact
// distance t (an upper bound of the true k-th) collected per query. The true
// top k is among them. Block = 128 rows x K2_RANGE_Q redo queries (held in
// shared memory); a query whose collection overflows K2_RANGE_CAP is left to
// the fp32 scan.
constexpr uint32_t K2_RANGE_Q = 4;
constexpr uint32_t K2_RANGE_CAP = 4096;
__global__ void __launch_bounds__(128) k2_range_kernel(const float* __restrict__ Qr, const float* __restrict__ thr,
                                                       uint32_t nredo, const float* __restrict__ rank_rows,
                                                       uint32_t nrank, uint32_t dim, int metric,
                                                       uint64_t* __restrict__ buf, uint32_t* __restrict__ cnt) {
  __shared__ float sq[K2_RANGE_Q][K2_MAX_DIM];
  const uint32_t q0 = blockIdx.y * K2_RANGE_Q;
  const uint32_t nqb = min(K2_RANGE_Q, nredo - q0);
  for (uint32_t e = threadIdx.x; e < nqb * dim; e += blockDim.x) sq[e / dim][e % dim] = Qr[(size_t)(q0 + e / dim) * dim + e % dim];
  __syncthreads();
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= nrank) return;
  const float* x = rank_rows + (size_t)r * dim;
  for (uint32_t j = 0; j < nqb; ++j) {
    const float d = k2_ref_distance(metric, sq[j], x, dim);
    const uint32_t key = order_key(d);
    if (key <= order_key(thr[q0 + j])) {
      const uint32_t pos = atomicAdd(cnt + q0 + j, 1u);
      if (pos < K2_RANGE_CAP) buf[(size_t)(q0 + j) * K2_RANGE_CAP + pos] = (static_cast<uint64_t>(key) << 32) | r;
    }
  }
}

// Per redo query: sort the collected (distance, rank) keys and write the first
// k to the query's result row; flag an overflow. 256 threads.
__global__ void __launch_bounds__(256) k2_range_finish_kernel(const uint64_t* __restrict__ buf,
                                                              const uint32_t* __restrict__ cnt,
                                                              const uint32_t* __restrict__ idx, uint32_t k,
                                                              const uint64_t* __restrict__ rank_id,
                                                              uint64_t* __restrict__ out_ids,
                                                              float* __restrict__ out_dist, uint32_t* __restrict__ out_len,
                                                              uint8_t* __restrict__ overflow) {
  extern __shared__ uint64_t sb[];  // [K2_RANGE_CAP]
  const uint32_t i = blockIdx.x;
  const uint32_t n = cnt[i];
  if (n > K2_RANGE_CAP) {
    if (threadIdx.x == 0) overflow[i] = 1;
    return;
  }
  uint32_t cap = 32;
  while (cap < n) cap <<= 1;
  for (uint32_t e = threadIdx.x; e < cap; e += blockDim.x) sb[e] = e < n ? buf[(size_t)i * K2_RANGE_CAP + e] : ~0ull;
  __syncthreads();
  block_bitonic_sort_u64(sb, cap);
  const uint32_t q = idx[i];
  const uint32_t take = min(n, k);
  for (uint32_t e = threadIdx.x; e < take; e += blockDim.x) {
    out_ids[(size_t)q * k + e] = rank_id[static_cast<uint32_t>(sb[e])];
    out_dist[(size_t)q * k + e] = key_to_float(static_cast<uint32_t>(sb[e] >> 32));
  }
  if (threadIdx.x == 0) {
    out_len[q] = take;
    overflow[i] = 0;
  }
}

__global__ void gather_f32_kernel(const float* __restrict__ src, const uint32_t* __restrict__ idx, uint32_t n,
                                  float* __restrict__ out) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = src[idx[i]];
}

}  // namespace pxc

using namespace pxc;

struct pxc_flat {
  pxc_ctx* ctx = nullptr;
  uint32_t dim = 0;
  int32_t metric = 0;
  uint64_t nslots = 0;  // mirror high-water mark
  DBuf<float> rows;
  DBuf<uint64_t> ids;
  DBuf<uint8_t> live;
  DBuf<uint8_t> rowflag;
  bool dirty = true;
  // rank mirror (live rows in ascending id order)
  uint64_t nrank = 0;
  DBuf<uint32_t> rank_slot;
  DBuf<uint64_t> rank_id;
  DBuf<float> rank_rows;
  bool all_u8 = false;
  uint32_t dp = 0;
  uint64_t nrank_pad = 0;
  DBuf<uint8_t> op_u8;
  DBuf<int32_t> op_norm;
  CUtensorMap tmap_x;
  // filtered K1: the operand of the accepted ranks only (rebuilt per search)
  DBuf<uint8_t> f_flags, f_op;
  DBuf<uint32_t> f_acc, f_count;
  DBuf<int32_t> f_norm;
  DBuf<uint64_t> f_id;
  // scratch
  DBuf<unsigned char> tmp;
  DBuf<uint32_t> dchunk;
  DBuf<uint64_t> lists_a, lists_b;
  DBuf<uint32_t> lens_a, lens_b;
  DBuf<uint8_t> q_u8;
  DBuf<int32_t> q_norm;
  DBuf<int> q_bad;
  DBuf<uint64_t> part;
  DBuf<int32_t> bound;
  DBuf<uint32_t> done;  // per query tile: finished-split counter, then the finished split ids
  DBuf<float> stage_f;
  DBuf<uint64_t> stage_id;
  DBuf<unsigned long long> bad_idx;
  // grouped K1 (32 < k <= 128): per-group lists, the queries searched again on K1g
  DBuf<uint64_t> g_ids, g_redo_ids;
  DBuf<float> g_dist, g_redo_q, g_redo_dist;
  DBuf<uint32_t> g_len, g_redo_idx, g_redo_len;
  DBuf<uint32_t> g_bound;  // [nq_pad] the sample pass's shared admission bound (packed keys)
  DBuf<uint64_t> c_cand;   // collect mode: [nq][nsplit][seg] candidate keys
  DBuf<uint32_t> c_cnt;    // collect mode: [nq][nsplit] candidates found
  DBuf<uint8_t> c_over;    // collect mode: [nq] the query's segments overflowed
  DBuf<uint32_t> c_idx, c_n, c_bound, c_len;  // the overflowed queries, gathered
  DBuf<float> c_q, c_dist;
  DBuf<uint64_t> c_ids;
  DBuf<uint8_t> g_redo;
  // buffers of the host-pointer entry point, kept across calls
  DBuf<float> io_q;
  DBuf<uint64_t> io_bm, io_ids;
  DBuf<float> io_dist;
  DBuf<uint32_t> io_len;
  // scan timing (profiling on): events around the dominant scan kernel
  cudaEvent_t ev_begin = nullptr, ev_end = nullptr;
  bool ev_recorded = false;
  int* h_flag = nullptr;  // pinned
  // This handle's device error word for K1's bounded waits ([0] code, [1] block)
  // and its pinned mirror: handles on one context search concurrently, so each
  // reads back only the failures of its own kernels.
  uint32_t* d_status = nullptr;
  uint32_t* h_status = nullptr;
  // K2 operand (built on the first non-integer search after the mirror changed)
  int k2_state = 0;  // 0: not built, 1: built, 2: not applicable to this store
  uint32_t k2_dp = 0;           // f16 elements per operand row (dim rounded up to 64)
  uint64_t k2_nrank_pad = 0;
  int k2_ax = 0;                // rows are scaled by 2^k2_ax
  DBuf<__half> k2_op, k2_q;
  DBuf<float> k2_h, k2_mu, k2_coef;
  DBuf<double> k2_part;
  DBuf<uint32_t> k2_stats;      // max |x'_i|, max ||x'||, max ||x||, max |h_x| (float bits)
  DBuf<K2Query> k2_meta;
  CUtensorMap k2_tmap_x;
  DBuf<float> k2_kth, k2_thr;     // per query: the candidates' k-th exact distance; gathered for redo queries
  DBuf<uint64_t> k2_range;        // [nredo][K2_RANGE_CAP] collected (distance, rank) keys
  DBuf<uint32_t> k2_range_cnt, k2_ovf_idx, k2_ovf_len;
  DBuf<uint8_t> k2_ovf;
  uint32_t last_redo = 0;  // queries of the last grouped search redone on K1g
  cudaEvent_t ev_done = nullptr;  // end of the last search's work (handoff of the scratch)
  std::mutex mu;
};

namespace {

// Events bracketing the scan kernel(s) of one search, when profiling is on.
struct ScanTimer {
  pxc_flat* h;
  cudaStream_t s;
  bool on;
  ScanTimer(pxc_flat* h_, cudaStream_t s_, bool enable = true) : h(h_), s(s_), on(enable && h_->ctx->profiling) {
    if (!on) return;
    if (!h->ev_begin) {
      PXC_CUDA(cudaEventCreate(&h->ev_begin));
      PXC_CUDA(cudaEventCreate(&h->ev_end));
    }
    PXC_CUDA(cudaEventRecord(h->ev_begin, s));
  }
  void stop() {
    if (!on) return;
    PXC_CUDA(cudaEventRecord(h->ev_end, s));
    h->ev_recorded = true;
  }
};

// The handle's device scratch and mirror pass from one call to the next in
// stream order. A search may return before its kernels finish (the fp32 scan
// does), and concurrent searches may run on different streams, so each search
// makes its stream wait (on the GPU) for the previous search's work, and
// records the end of its own; calls that rewrite the mirror wait on the host.
void handoff_wait(pxc_flat* h, cudaStream_t s) {
  if (h->ev_done) PXC_CUDA(cudaStreamWaitEvent(s, h->ev_done, 0));
}
void handoff_done(pxc_flat* h, cudaStream_t s) {
  if (!h->ev_done) PXC_CUDA(cudaEventCreateWithFlags(&h->ev_done, cudaEventDisableTiming));
  PXC_CUDA(cudaEventRecord(h->ev_done, s));
}
void handoff_drain(pxc_flat* h) {
  if (h->ev_done) PXC_CUDA(cudaEventSynchronize(h->ev_done));
}

void ensure_capacity(pxc_flat* h, uint64_t want, cudaStream_t s) {
  uint64_t cap = h->ids.n;
  if (want <= cap) return;
  uint64_t ncap = std::max<uint64_t>(want, cap + cap / 2);
  ncap = std::max<uint64_t>(ncap, 1024);
  h->rows.grow_keep(ncap * h->dim, h->nslots * h->dim, s);
  h->ids.grow_keep(ncap, h->nslots, s);
  h->live.grow_keep(ncap, h->nslots, s);
  h->rowflag.grow_keep(ncap, h->nslots, s);
}

void rebuild_mirror(pxc_flat* h, cudaStream_t s) {
  const uint64_t n = h->nslots;
  h->nrank = 0;
  h->all_u8 = false;
  h->k2_state = 0;
  if (n == 0) {
    h->dirty = false;
    return;
  }
  PXC_CONFIG(n < (1ull << 32), "slots", n, "the device mirror addresses at most 2^32 slots");
  // 1. live slots in slot order
  DBuf<uint32_t> slots_all, slots_live, sorted_slots;
  DBuf<uint64_t> keys, sorted_keys;
  DBuf<int> num;
  slots_all.reserve(n);
  slots_live.reserve(n);
  num.reserve(2);
  iota_u32_kernel<<<grid1d(n, 256), 256, 0, s>>>(slots_all.p, n);
  size_t tb = 0;
  PXC_CUDA(cub::DeviceSelect::Flagged(nullptr, tb, slots_all.p, h->live.p, slots_live.p, num.p, (int64_t)n, s));
  h->tmp.reserve(tb);
  PXC_CUDA(cub::DeviceSelect::Flagged(h->tmp.p, tb, slots_all.p, h->live.p, slots_live.p, num.p, (int64_t)n, s));
  PXC_CUDA(cudaMemcpyAsync(h->h_flag, num.p, sizeof(int), cudaMemcpyDeviceToHost, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  const uint64_t nl = static_cast<uint64_t>(*h->h_flag);
  h->nrank = nl;
  if (nl == 0) {
    h->dirty = false;
    return;
  }
  // 2. sort live slots by id
  keys.reserve(nl);
  sorted_keys.reserve(nl);
  sorted_slots.reserve(nl);
  gather_ids_kernel<<<grid1d(nl, 256), 256, 0, s>>>(slots_live.p, h->ids.p, keys.p, nl);
  tb = 0;
  PXC_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tb, keys.p, sorted_keys.p, slots_live.p,
                                           sorted_slots.p, (int64_t)nl, 0, 64, s));
  h->tmp.reserve(tb);
  PXC_CUDA(cub::DeviceRadixSort::SortPairs(h->tmp.p, tb, keys.p, sorted_keys.p, slots_live.p,
                                           sorted_slots.p, (int64_t)nl, 0, 64, s));
  h->rank_slot.reserve(nl);
  h->rank_id.reserve(nl);
  PXC_CUDA(cudaMemcpyAsync(h->rank_slot.p, sorted_slots.p, nl * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s));
  PXC_CUDA(cudaMemcpyAsync(h->rank_id.p, sorted_keys.p, nl * sizeof(uint64_t), cudaMemcpyDeviceToDevice, s));
  // 3. rank-ordered rows and the u8 classification
  h->rank_rows.reserve(nl * h->dim);
  PXC_CUDA(cudaMemsetAsync(num.p, 0xFF, sizeof(int), s));
  gather_rows_kernel<<<(unsigned)nl, 128, 0, s>>>(h->rank_slot.p, h->rows.p, h->rowflag.p, h->dim,
                                                  h->rank_rows.p, num.p);
  PXC_CUDA(cudaGetLastError());
  PXC_CUDA(cudaMemcpyAsync(h->h_flag, num.p, sizeof(int), cudaMemcpyDeviceToHost, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  h->all_u8 = (*h->h_flag != 0);
  // 4. u8 operand for the tensor-core path
  if (h->all_u8 && h->metric == PXC_EUCLIDEAN && h->dim <= (uint32_t)flat_tc::MAX_KBLOCKS * flat_tc::KB_BYTES) {
    h->dp = (h->dim + 127) / 128 * 128;
    h->nrank_pad = (nl + flat_tc::BN - 1) / flat_tc::BN * flat_tc::BN;
    h->op_u8.reserve(h->nrank_pad * h->dp);
    h->op_norm.reserve(h->nrank_pad);
    build_u8_operand_kernel<<<(unsigned)h->nrank_pad, 128, 0, s>>>(h->rank_rows.p, nl, h->dim, h->dp,
                                                                  h->op_u8.p, h->op_norm.p);
    PXC_CUDA(cudaGetLastError());
    make_tmap_u8_2d(&h->tmap_x, h->op_u8.p, h->dp, h->nrank_pad, flat_tc::KB_BYTES, flat_tc::BN);
  }
  PXC_CUDA(cudaStreamSynchronize(s));
  h->dirty = false;
}

// Number of row splits for K1: balance waves of CTAs over the SMs.
// At most 2048 / KT splits, so one query's candidates fit the merge block.
uint32_t choose_splits(uint32_t nqt, uint32_t ntiles, int sms, uint32_t KT) {
  uint32_t smax = std::max<uint32_t>(1, std::min<uint32_t>(ntiles / 8, 2048 / KT));
  double best = 1e30;
  uint32_t best_s = 1;
  for (uint32_t s = 1; s <= smax; ++s) {
    uint32_t tps = (ntiles + s - 1) / s;
    uint32_t ctas = nqt * ((ntiles + tps - 1) / tps);
    double waves = std::ceil((double)ctas / sms);
    // +10 tiles of fixed per-CTA cost; the first wave starts without seeds
    // from finished splits and runs about 1.5x slower, hence the 0.5/waves.
    double cost = waves * (tps + 10.0) * (1.0 + 0.5 / waves);
    if (cost < best * 0.995) {
      best = cost;
      best_s = s;
    }
  }
  return best_s;
}

template <int KT, class P = flat_tc::U8Scan, bool COLLECT = false>
void launch_tc(const CUtensorMap& tq, const CUtensorMap& tx, const flat_tc::Params& p, dim3 grid,
               size_t smem, cudaStream_t s) {
  PXC_CUDA(cudaFuncSetAttribute(flat_tc::flat_scan_kernel<KT, P, COLLECT>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  flat_tc::flat_scan_kernel<KT, P, COLLECT><<<grid, flat_tc::NUM_THREADS, smem, s>>>(tq, tx, p);
}

// The database side of one K1 search: the full mirror, or the accepted ranks of a filter.
struct TcOperand {
  const CUtensorMap* tmap_x;
  const int32_t* norms;
  uint64_t nrank_pad;
  const uint64_t* rank_id;
  uint64_t nrank;
  const uint8_t* rows;  // [nrank_pad][dp] u8, the memory tmap_x describes
};

// One K1 search of nq queries over op. init_bound (optional, [nq_pad] packed
// keys) replaces the "no bound yet" start of the shared admission bound.
void search_tc(pxc_flat* h, const TcOperand& op, const float* d_q, uint32_t nq, uint32_t k, uint64_t* d_ids,
               float* d_dist, uint32_t* d_len, cudaStream_t s, bool timed = true,
               const uint32_t* init_bound = nullptr) {
  const uint32_t KT = k <= 1 ? 1 : k <= 4 ? 4 : k <= 10 ? 10 : k <= 16 ? 16 : 32;
  const uint32_t nq_pad = (nq + flat_tc::BM - 1) / flat_tc::BM * flat_tc::BM;
  const uint32_t nqt = nq_pad / flat_tc::BM;
  const uint32_t ntiles = (uint32_t)(op.nrank_pad / flat_tc::BN);
  const uint32_t nsplit_req = choose_splits(nqt, ntiles, h->ctx->sm_count, KT);
  const uint32_t tps = (ntiles + nsplit_req - 1) / nsplit_req;
  const uint32_t nsplit = (ntiles + tps - 1) / tps;
  h->part.reserve((size_t)nq_pad * nsplit * KT);
  h->bound.reserve(nq_pad);
  h->done.reserve(nqt + (size_t)nqt * nsplit);
  // 0x3F3F3F3F: above every real r (|r| < 2^25) and below the padding sentinel
  if (init_bound != nullptr)
    PXC_CUDA(cudaMemcpyAsync(h->bound.p, init_bound, nq_pad * sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
  else
    PXC_CUDA(cudaMemsetAsync(h->bound.p, 0x3F, nq_pad * sizeof(int32_t), s));
  PXC_CUDA(cudaMemsetAsync(h->done.p, 0, nqt * sizeof(uint32_t), s));
  PXC_CUDA(cudaMemsetAsync(h->done.p + nqt, 0xFF, (size_t)nqt * nsplit * sizeof(uint32_t), s));
  flat_tc::Params p;
  p.norms = op.norms;
  p.qcoef = nullptr;
  p.qdelta = nullptr;
  p.bound = reinterpret_cast<uint32_t*>(h->bound.p);
  p.done_count = h->done.p;
  p.done_list = h->done.p + nqt;
  p.out_part = h->part.p;
  p.status = h->d_status;
  p.nq = nq;
  p.k = k;
  p.kblocks = h->dp / flat_tc::KB_BYTES;
  p.ntiles = ntiles;
  p.tiles_per_split = tps;
  p.nsplit = nsplit;
  p.stages = flat_tc::pick_stages<flat_tc::U8Scan>(p.kblocks);
  p.wait_ns = (uint64_t)h->ctx->wait_ms * 1000000ull;
  CUtensorMap tmap_q;
  make_tmap_u8_2d(&tmap_q, h->q_u8.p, h->dp, nq_pad, flat_tc::KB_BYTES, flat_tc::BM);
  size_t smem = flat_tc::smem_bytes<flat_tc::U8Scan>(p.kblocks, p.stages);
  dim3 grid(nqt, nsplit);
  ScanTimer timer(h, s, timed);
  switch (KT) {
    case 1: launch_tc<1>(tmap_q, *op.tmap_x, p, grid, smem, s); break;
    case 4: launch_tc<4>(tmap_q, *op.tmap_x, p, grid, smem, s); break;
    case 10: launch_tc<10>(tmap_q, *op.tmap_x, p, grid, smem, s); break;
    case 16: launch_tc<16>(tmap_q, *op.tmap_x, p, grid, smem, s); break;
    default: launch_tc<32>(tmap_q, *op.tmap_x, p, grid, smem, s); break;
  }
  PXC_CUDA(cudaGetLastError());
  timer.stop();
  h->ctx->launches += 2;  // scan + merge
  uint32_t cap = 32;
  while (cap < nsplit * KT) cap <<= 1;
  size_t msmem = cap * sizeof(uint64_t);
  if (msmem > 48 * 1024)
    PXC_CUDA(cudaFuncSetAttribute(merge_u8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msmem));
  merge_u8_kernel<<<nq, 256, msmem, s>>>(h->part.p, nsplit, KT, cap, k, h->q_norm.p, op.rank_id, (uint32_t)op.nrank,
                                         d_ids, d_dist, d_len, nullptr);
  PXC_CUDA(cudaGetLastError());
}

template <int METRIC>
void launch_dist(const float* d_q, uint32_t nqb, const pxc_flat* h, uint64_t c0, uint32_t C,
                 const uint64_t* bitmap, uint32_t* D, cudaStream_t s) {
  dim3 grid(C / 64, (nqb + 31) / 32);
  dist_chunk_kernel<METRIC><<<grid, 256, 0, s>>>(d_q, nqb, h->rank_rows.p, h->nrank, h->dim, c0, C,
                                                 bitmap, h->rank_slot.p, D);
}

void search_generic(pxc_flat* h, const float* d_q, uint32_t nq, uint32_t k, const uint64_t* d_bitmap,
                    uint64_t* d_ids, float* d_dist, uint32_t* d_len, cudaStream_t s) {
  const uint64_t nrank = h->nrank;
  const uint64_t list_budget = 1ull << 26;  // entries per list buffer (512 MiB)
  const uint32_t qbatch = (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(nq, std::min<uint64_t>(65536, list_budget / k)));
  const uint64_t dbudget = 1ull << 26;  // chunk keys (256 MiB)
  uint64_t C64 = std::max<uint64_t>(64, dbudget / qbatch / 64 * 64);
  uint64_t nr64 = (nrank + 63) / 64 * 64;
  const uint32_t C = (uint32_t)std::min<uint64_t>(C64, nr64);
  h->dchunk.reserve((size_t)qbatch * C);
  h->lists_a.reserve((size_t)qbatch * k);
  h->lists_b.reserve((size_t)qbatch * k);
  h->lens_a.reserve(qbatch);
  h->lens_b.reserve(qbatch);
  ScanTimer timer(h, s);
  for (uint32_t qb = 0; qb < nq; qb += qbatch) {
    const uint32_t nqb = std::min(qbatch, nq - qb);
    const float* q = d_q + (size_t)qb * h->dim;
    uint64_t* La = h->lists_a.p;
    uint64_t* Lb = h->lists_b.p;
    uint32_t* la = h->lens_a.p;
    uint32_t* lb = h->lens_b.p;
    zero_u32_kernel<<<grid1d(nqb, 256), 256, 0, s>>>(la, nqb);
    for (uint64_t c0 = 0; c0 < nrank; c0 += C) {
      const uint32_t cvalid = (uint32_t)std::min<uint64_t>(C, nrank - c0);
      switch (h->metric) {
        case PXC_EUCLIDEAN: launch_dist<PXC_EUCLIDEAN>(q, nqb, h, c0, C, d_bitmap, h->dchunk.p, s); break;
        case PXC_COSINE: launch_dist<PXC_COSINE>(q, nqb, h, c0, C, d_bitmap, h->dchunk.p, s); break;
        case PXC_INNER_PRODUCT: launch_dist<PXC_INNER_PRODUCT>(q, nqb, h, c0, C, d_bitmap, h->dchunk.p, s); break;
        default: launch_dist<PXC_MANHATTAN>(q, nqb, h, c0, C, d_bitmap, h->dchunk.p, s); break;
      }
      PXC_CUDA(cudaGetLastError());
      select_chunk_kernel<<<nqb, SEL_THREADS, 0, s>>>(La, la, Lb, lb, h->dchunk.p, C, c0, cvalid, k, 0);
      PXC_CUDA(cudaGetLastError());
      h->ctx->launches += 2;
      std::swap(La, Lb);
      std::swap(la, lb);
    }
    h->ctx->launches += 2;  // list reset + finalize
    if (k <= 2048) {
      uint32_t cap = 32;
      while (cap < k) cap <<= 1;
      size_t smem = cap * sizeof(uint64_t);
      if (smem > 48 * 1024)
        PXC_CUDA(cudaFuncSetAttribute(finalize_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      finalize_small_kernel<<<nqb, 256, smem, s>>>(La, la, k, cap, h->rank_id.p, qb, d_ids, d_dist, d_len);
    } else {
      pad_lists_kernel<<<nqb, 256, 0, s>>>(La, la, k);
      std::vector<int64_t> offs(nqb + 1);
      for (uint32_t i = 0; i <= nqb; ++i) offs[i] = (int64_t)i * k;
      DBuf<int64_t> d_offs;
      d_offs.reserve(nqb + 1);
      PXC_CUDA(cudaMemcpyAsync(d_offs.p, offs.data(), (nqb + 1) * sizeof(int64_t), cudaMemcpyHostToDevice, s));
      size_t tb = 0;
      PXC_CUDA(cub::DeviceSegmentedRadixSort::SortKeys(nullptr, tb, La, Lb, (int64_t)nqb * k, (int64_t)nqb,
                                                      d_offs.p, d_offs.p + 1, 0, 64, s));
      h->tmp.reserve(tb);
      PXC_CUDA(cub::DeviceSegmentedRadixSort::SortKeys(h->tmp.p, tb, La, Lb, (int64_t)nqb * k, (int64_t)nqb,
                                                      d_offs.p, d_offs.p + 1, 0, 64, s));
      finalize_sorted_kernel<<<nqb, 256, 0, s>>>(Lb, la, k, h->rank_id.p, qb, d_ids, d_dist, d_len);
      PXC_CUDA(cudaStreamSynchronize(s));  // d_offs is freed on return
    }
    PXC_CUDA(cudaGetLastError());
  }
  timer.stop();
}

// 32 < k <= 128 on the tensor cores: the operand is cut into groups of whole
// 256-row tiles, K1 returns each group's top GROUP_K, the group lists are
// merged by (distance, id), and group_check_kernel proves the merged top k
// exact per query; the few queries it cannot prove are searched again on K1g.
// Groups: ceil(0.08 k), so a group holds 1/12.5 of a query's top k on
// average and reaching GROUP_K in one group is rare unless rows that are near
// one another are also near in id order.
//
// Every launch below starts from one admission bound T per query instead of
// "no bound": a sample pass runs one K1 launch for the top SAMPLE_K over
// about k / SAMPLE_TARGET of the rows, in ns = ceil(2k / SAMPLE_K) runs of
// tiles spread evenly over the operand (one split each, keeping its own list:
// Params::share = 0, no seeding, no shared bound), and T is the k-th smallest
// r of the union of those lists. The
// splits cover disjoint rows, so at least k distinct rows have r <= T, the
// true k-th has r <= T, and a row turned away at T (r > T) is behind it. The
// proof above is unchanged: a group list that is not full holds every row of
// its group with r <= T.
constexpr uint32_t SAMPLE_K = 16;
constexpr uint32_t SAMPLE_TARGET = 800;  // rows of the operand per row of the sample's top k (k x divisor)
constexpr uint32_t SAMPLE_MAX = 256;  // union entries per query: ns * SAMPLE_K <= 256 for k <= 128

// T per query from the sample launch's lists ([nq_pad][nsplit][SAMPLE_K]
// packed (r, rank) keys): the k-th smallest r key of the union, or "no bound"
// (0x3F3F3F3F) when the lists hold fewer than k rows or q >= nq. One block of
// SAMPLE_MAX threads per query (nq_pad blocks), nsplit * SAMPLE_K <= SAMPLE_MAX.
__global__ void __launch_bounds__(SAMPLE_MAX) union_kth_kernel(const uint64_t* __restrict__ part, uint32_t nsplit,
                                                               uint32_t nq, uint32_t k, uint32_t* __restrict__ T) {
  __shared__ uint32_t key[SAMPLE_MAX];
  __shared__ uint32_t total;
  const uint32_t q = blockIdx.x;
  if (q >= nq) {
    if (threadIdx.x == 0) T[q] = 0x3F3F3F3Fu;
    return;
  }
  if (threadIdx.x == 0) total = 0;
  const uint32_t n = nsplit * SAMPLE_K;
  const uint32_t empty = flat_tc::U8Scan::pack(flat_tc::BIG);
  uint32_t v = 0xFFFFFFFFu;
  if (threadIdx.x < n) {
    const uint32_t r = static_cast<uint32_t>(part[(size_t)q * n + threadIdx.x] >> 32);
    if (r < empty) v = r;
  }
  key[threadIdx.x] = v;
  __syncthreads();
  if (v != 0xFFFFFFFFu) atomicAdd(&total, 1u);
  for (uint32_t size = 2; size <= SAMPLE_MAX; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      const uint32_t i = threadIdx.x, o = i ^ stride;
      if (o > i) {
        const uint32_t a = key[i], b = key[o];
        const bool up = (i & size) == 0;
        if ((a > b) == up) {
          key[i] = b;
          key[o] = a;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) T[q] = total < k ? 0x3F3F3F3Fu : key[k - 1];
}

// The sample pass: one K1 launch (KT = SAMPLE_K, share = 0) in ns splits of
// stiles tiles, split i starting at tile i * (ntiles / ns), then
// union_kth_kernel into T [nq_pad].
void sample_bound(pxc_flat* h, const TcOperand& op, uint32_t nq, uint32_t k, uint32_t ns, uint32_t stiles,
                  uint32_t* T, cudaStream_t s) {
  const uint32_t nq_pad = (nq + flat_tc::BM - 1) / flat_tc::BM * flat_tc::BM;
  const uint32_t nqt = nq_pad / flat_tc::BM;
  h->part.reserve((size_t)nq_pad * ns * SAMPLE_K);
  h->bound.reserve(nq_pad);
  h->done.reserve(nqt + (size_t)nqt * ns);
  PXC_CUDA(cudaMemsetAsync(h->bound.p, 0x3F, nq_pad * sizeof(int32_t), s));
  PXC_CUDA(cudaMemsetAsync(h->done.p, 0, nqt * sizeof(uint32_t), s));
  PXC_CUDA(cudaMemsetAsync(h->done.p + nqt, 0xFF, (size_t)nqt * ns * sizeof(uint32_t), s));
  flat_tc::Params p;
  p.norms = op.norms;
  p.qcoef = nullptr;
  p.qdelta = nullptr;
  p.bound = reinterpret_cast<uint32_t*>(h->bound.p);
  p.done_count = h->done.p;
  p.done_list = h->done.p + nqt;
  p.out_part = h->part.p;
  p.share = 0;
  p.status = h->d_status;
  p.nq = nq;
  p.k = SAMPLE_K;
  p.kblocks = h->dp / flat_tc::KB_BYTES;
  p.ntiles = (uint32_t)(op.nrank_pad / flat_tc::BN);
  p.tiles_per_split = stiles;  // <= ntiles / ns, so the runs do not overlap
  p.split_stride = p.ntiles / ns;
  p.nsplit = ns;
  p.stages = flat_tc::pick_stages<flat_tc::U8Scan>(p.kblocks);
  p.wait_ns = (uint64_t)h->ctx->wait_ms * 1000000ull;
  CUtensorMap tmap_q;
  make_tmap_u8_2d(&tmap_q, h->q_u8.p, h->dp, nq_pad, flat_tc::KB_BYTES, flat_tc::BM);
  const size_t smem = flat_tc::smem_bytes<flat_tc::U8Scan>(p.kblocks, p.stages);
  launch_tc<SAMPLE_K>(tmap_q, *op.tmap_x, p, dim3(nqt, ns), smem, s);
  PXC_CUDA(cudaGetLastError());
  union_kth_kernel<<<nq_pad, SAMPLE_MAX, 0, s>>>(h->part.p, ns, nq, k, T);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 2;
}


constexpr uint64_t COLLECT_MAX_ENTRIES = 1ull << 26;  // collect-mode candidate slots per search (512 MiB)

// Collect mode (32 < k <= 128 once the sample pass has given T): ONE K1
// launch over the whole operand with the fixed starting bound T appends every
// (r, rank) with r <= T to the query's candidate row (cap slots), and the
// merge sorts the filled prefix and keeps k. Every row of the true top k has
// r <= T, so the result is exact for every query whose row did not overflow;
// those that did are flagged in redo.
__global__ void overflow_flags_kernel(const uint32_t* __restrict__ cnt, uint32_t nq, uint32_t nsplit, uint32_t seg,
                                      uint32_t cap, uint8_t* __restrict__ redo) {
  const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  uint32_t total = 0;
  bool over = false;
  for (uint32_t sp = 0; sp < nsplit; ++sp) {
    const uint32_t c = cnt[(size_t)q * nsplit + sp];
    over |= c > seg;
    total += min(c, seg);
  }
  redo[q] = (over || total > cap) ? 1 : 0;
}

// Slots per (query, split) segment: twice an even share of the query's cap,
// a power of two in [256, cap].
inline uint32_t collect_segment(uint32_t cap, uint32_t nsplit) {
  uint32_t seg = 256;
  while (seg < cap && seg * nsplit < 2 * cap) seg <<= 1;
  return std::min(seg, cap);
}

// Returns false (nothing launched) when the segments would exceed
// COLLECT_MAX_ENTRIES slots.
bool search_tc_collect(pxc_flat* h, const TcOperand& op, uint32_t nq, uint32_t k, const uint32_t* T, uint32_t cap,
                       uint64_t* d_ids, float* d_dist, uint32_t* d_len, uint8_t* redo, cudaStream_t s) {
  const uint32_t nq_pad = (nq + flat_tc::BM - 1) / flat_tc::BM * flat_tc::BM;
  const uint32_t nqt = nq_pad / flat_tc::BM;
  const uint32_t ntiles = (uint32_t)(op.nrank_pad / flat_tc::BN);
  // choose_splits with KT 32 keeps nsplit <= 2048 / 32 = MERGE_MAX_SPLITS
  const uint32_t nsplit_req = choose_splits(nqt, ntiles, h->ctx->sm_count, 32);
  const uint32_t tps = (ntiles + nsplit_req - 1) / nsplit_req;
  const uint32_t nsplit = (ntiles + tps - 1) / tps;
  const uint32_t seg = collect_segment(cap, nsplit);
  if ((uint64_t)nq * nsplit * seg > COLLECT_MAX_ENTRIES) return false;
  h->c_cand.reserve((size_t)nq * nsplit * seg);
  h->c_cnt.reserve((size_t)nq * nsplit);
  h->bound.reserve(nq_pad);
  h->done.reserve(nqt + (size_t)nqt * nsplit);
  PXC_CUDA(cudaMemcpyAsync(h->bound.p, T, nq_pad * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s));
  PXC_CUDA(cudaMemsetAsync(h->done.p, 0, nqt * sizeof(uint32_t), s));
  PXC_CUDA(cudaMemsetAsync(h->done.p + nqt, 0xFF, (size_t)nqt * nsplit * sizeof(uint32_t), s));
  flat_tc::Params p;
  p.norms = op.norms;
  p.qcoef = nullptr;
  p.qdelta = nullptr;
  p.bound = reinterpret_cast<uint32_t*>(h->bound.p);
  p.done_count = h->done.p;
  p.done_list = h->done.p + nqt;
  p.out_part = nullptr;
  p.cand = h->c_cand.p;
  p.cand_cnt = h->c_cnt.p;
  p.cand_cap = seg;
  p.status = h->d_status;
  p.nq = nq;
  p.k = 1;  // the (empty) list never publishes: the bound stays T
  p.kblocks = h->dp / flat_tc::KB_BYTES;
  p.ntiles = ntiles;
  p.tiles_per_split = tps;
  p.nsplit = nsplit;
  p.stages = flat_tc::pick_stages<flat_tc::U8Scan>(p.kblocks);
  p.wait_ns = (uint64_t)h->ctx->wait_ms * 1000000ull;
  CUtensorMap tmap_q;
  make_tmap_u8_2d(&tmap_q, h->q_u8.p, h->dp, nq_pad, flat_tc::KB_BYTES, flat_tc::BM);
  const size_t smem = flat_tc::smem_bytes<flat_tc::U8Scan>(p.kblocks, p.stages);
  launch_tc<1, flat_tc::U8Scan, true>(tmap_q, *op.tmap_x, p, dim3(nqt, nsplit), smem, s);
  PXC_CUDA(cudaGetLastError());
  merge_u8_kernel<<<nq, 256, cap * sizeof(uint64_t), s>>>(h->c_cand.p, nsplit, seg, cap, k, h->q_norm.p, op.rank_id,
                                                           (uint32_t)op.nrank, d_ids, d_dist, d_len, h->c_cnt.p);
  PXC_CUDA(cudaGetLastError());
  overflow_flags_kernel<<<grid1d(nq, 256), 256, 0, s>>>(h->c_cnt.p, nq, nsplit, seg, cap, redo);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 3;  // scan + merge + flags
  return true;
}

// Queries of a 0/1 flag array ([n]) as an index list; returns how many.
uint32_t flagged_queries(pxc_flat* h, const uint8_t* flags, uint32_t n, uint32_t* idx, uint32_t* count,
                         cudaStream_t s) {
  size_t tb = 0;
  thrust::counting_iterator<uint32_t> it(0);
  PXC_CUDA(cub::DeviceSelect::Flagged(nullptr, tb, it, flags, idx, count, (int64_t)n, s));
  h->tmp.reserve(std::max<size_t>(tb, 1));
  PXC_CUDA(cub::DeviceSelect::Flagged(h->tmp.p, tb, it, flags, idx, count, (int64_t)n, s));
  PXC_CUDA(cudaMemcpyAsync(h->h_flag, count, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  h->ctx->launches += 2;  // two select passes
  return static_cast<uint32_t>(*h->h_flag);
}

// The group launches (K1 per group of tiles, starting from the bound T when
// given), the merge, the proof, and K1g for the queries it cannot prove.
// h->q_u8 / q_norm hold the queries d_q; sets h->last_redo to the K1g count.
void group_launches(pxc_flat* h, const TcOperand& op, const float* d_q, uint32_t nq, uint32_t k,
                    const uint32_t* shared_t, const uint64_t* d_bitmap, uint64_t* d_ids, float* d_dist,
                    uint32_t* d_len, cudaStream_t s) {
  const uint64_t ntiles = op.nrank_pad / flat_tc::BN;
  const uint32_t want = std::max<uint32_t>(2, (k * 2 + 24) / 25);
  const uint64_t tpg = (ntiles + want - 1) / want;
  const uint32_t ng = (uint32_t)((ntiles + tpg - 1) / tpg);
  h->g_ids.reserve((size_t)ng * nq * GROUP_K);
  h->g_dist.reserve((size_t)ng * nq * GROUP_K);
  h->g_len.reserve((size_t)ng * nq);
  h->g_redo.reserve(nq);
  h->g_redo_idx.reserve(nq);
  h->g_redo_len.reserve(1);  // the count first; resized below if queries need K1g
  for (uint32_t g = 0; g < ng; ++g) {
    const uint64_t t0 = (uint64_t)g * tpg;
    const uint64_t t1 = std::min<uint64_t>(ntiles, t0 + tpg);
    const uint64_t r0 = t0 * flat_tc::BN;
    const uint64_t rows_pad = (t1 - t0) * flat_tc::BN;
    // r0 < nrank: the last tile of the operand holds at least one real row
    const uint64_t nreal = std::min<uint64_t>(op.nrank, t1 * flat_tc::BN) - r0;
    CUtensorMap tm;
    make_tmap_u8_2d(&tm, op.rows + r0 * h->dp, h->dp, rows_pad, flat_tc::KB_BYTES, flat_tc::BN);
    TcOperand gop{&tm, op.norms + r0, rows_pad, op.rank_id + r0, nreal, op.rows + r0 * h->dp};
    const size_t off = (size_t)g * nq;
    search_tc(h, gop, d_q, nq, GROUP_K, h->g_ids.p + off * GROUP_K, h->g_dist.p + off * GROUP_K,
              h->g_len.p + off, s, false, shared_t);
  }
  pxc_error err{};
  if (pxc_topk_merge(h->ctx, h->g_ids.p, h->g_dist.p, h->g_len.p, ng, nq, GROUP_K, k, d_ids, d_dist, d_len, s,
                     &err) != PXC_OK)
    throw make_failure((pxc_status)err.code, err.a, err.b, nullptr, "group merge: %s", err.detail);
  group_check_kernel<<<grid1d(nq, 256), 256, 0, s>>>(h->g_ids.p, h->g_dist.p, h->g_len.p, ng, nq, d_ids, d_dist,
                                                      d_len, k, h->g_redo.p);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 1;
  const uint32_t nredo = flagged_queries(h, h->g_redo.p, nq, h->g_redo_idx.p, h->g_redo_len.p, s);
  h->last_redo = nredo;
  if (nredo == 0) return;
  h->g_redo_q.reserve((size_t)nredo * h->dim);
  h->g_redo_ids.reserve((size_t)nredo * k);
  h->g_redo_dist.reserve((size_t)nredo * k);
  h->g_redo_len.reserve(nredo);
  gather_queries_kernel<<<nredo, 128, 0, s>>>(d_q, h->g_redo_idx.p, h->dim, h->g_redo_q.p);
  PXC_CUDA(cudaGetLastError());
  search_generic(h, h->g_redo_q.p, nredo, k, d_bitmap, h->g_redo_ids.p, h->g_redo_dist.p, h->g_redo_len.p, s);
  scatter_results_kernel<<<nredo, 128, 0, s>>>(h->g_redo_ids.p, h->g_redo_dist.p, h->g_redo_len.p,
                                               h->g_redo_idx.p, k, d_ids, d_dist, d_len);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 2;
}

// Entry i of out = T[idx[i]] for i < n, "no bound" for n <= i < n_pad.
__global__ void gather_bound_kernel(const uint32_t* __restrict__ T, const uint32_t* __restrict__ idx, uint32_t n,
                                    uint32_t n_pad, uint32_t* __restrict__ out) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n_pad) out[i] = i < n ? T[idx[i]] : 0x3F3F3F3Fu;
}

// The sample is 1/divisor of the rows: SAMPLE_TARGET / k, or the diagnostic
// option's value when it is set (0: no sample pass).
uint64_t sample_divisor(const pxc_ctx* ctx, uint32_t k) {
  if (ctx->opt_flat_group_sample >= 0) return (uint64_t)ctx->opt_flat_group_sample;
  return std::max<uint64_t>(2, SAMPLE_TARGET / k);
}

// Query batches larger than this run in chunks, so that the collect launch's
// segments (up to 2 x 2,048 slots per query) stay within COLLECT_MAX_ENTRIES.
// Measured on C2 at k = 100: 10,000 queries as 8,192 + 1,808 take 5.33 ms,
// in one piece 6.23 ms, in chunks of 4,096 5.90 ms.
constexpr uint32_t GROUPED_CHUNK_Q = 8192;

void search_tc_grouped(pxc_flat* h, const TcOperand& op, const float* d_q, uint32_t nq, uint32_t k,
                       const uint64_t* d_bitmap, uint64_t* d_ids, float* d_dist, uint32_t* d_len, cudaStream_t s,
                       bool timed = true) {
  if (nq > GROUPED_CHUNK_Q) {
    ScanTimer timer(h, s, timed);  // all chunks
    uint32_t redone = 0;
    for (uint32_t q0 = 0; q0 < nq; q0 += GROUPED_CHUNK_Q) {
      const uint32_t n = std::min(GROUPED_CHUNK_Q, nq - q0);
      const uint32_t np = (n + flat_tc::BM - 1) / flat_tc::BM * flat_tc::BM;
      const float* q = d_q + (size_t)q0 * h->dim;
      // this chunk's u8 queries and norms at the front of the query buffers
      prep_queries_u8_kernel<<<np, 128, 0, s>>>(q, n, h->dim, h->dp, h->q_u8.p, h->q_norm.p, h->q_bad.p);
      PXC_CUDA(cudaGetLastError());
      h->ctx->launches += 1;
      search_tc_grouped(h, op, q, n, k, d_bitmap, d_ids + (size_t)q0 * k, d_dist + (size_t)q0 * k, d_len + q0, s,
                        false);
      redone += h->last_redo;
    }
    timer.stop();
    h->last_redo = redone;
    return;
  }
  const uint64_t ntiles = op.nrank_pad / flat_tc::BN;
  const uint32_t want = std::max<uint32_t>(2, (k * 2 + 24) / 25);
  if (ntiles < want) {  // too few rows to split: the fp32 scan
    search_generic(h, d_q, nq, k, d_bitmap, d_ids, d_dist, d_len, s);
    return;
  }
  ScanTimer timer(h, s, timed);
  const uint32_t* shared_t = nullptr;
  const uint64_t ns = (2 * k + SAMPLE_K - 1) / SAMPLE_K;  // <= SAMPLE_MAX / SAMPLE_K for k <= 128
  const uint64_t sdiv = sample_divisor(h->ctx, k);
  const uint64_t stiles = sdiv > 0 ? ntiles / sdiv / ns : 0;  // tiles per sample split
  if (stiles >= 1) {
    const uint32_t nq_pad = (nq + flat_tc::BM - 1) / flat_tc::BM * flat_tc::BM;
    h->g_bound.reserve(nq_pad);
    sample_bound(h, op, nq, k, (uint32_t)ns, (uint32_t)stiles, h->g_bound.p, s);
    shared_t = h->g_bound.p;
  }
  const uint64_t cap = (uint64_t)h->ctx->opt_flat_collect_cap;
  h->c_over.reserve(nq);
  if (shared_t == nullptr || cap < 32 ||
      !search_tc_collect(h, op, nq, k, shared_t, (uint32_t)cap, d_ids, d_dist, d_len, h->c_over.p, s)) {
    group_launches(h, op, d_q, nq, k, shared_t, d_bitmap, d_ids, d_dist, d_len, s);
    timer.stop();
    return;
  }
  timer.stop();
  // Queries whose candidate segments overflowed: the group launches, from
  // their own (valid, if loose) T, on the gathered queries.
  h->c_idx.reserve(nq);
  h->c_n.reserve(1);
  const uint32_t nover = flagged_queries(h, h->c_over.p, nq, h->c_idx.p, h->c_n.p, s);
  h->last_redo = 0;
  if (nover == 0) return;
  const uint32_t np = (nover + flat_tc::BM - 1) / flat_tc::BM * flat_tc::BM;
  h->c_q.reserve((size_t)nover * h->dim);
  h->c_ids.reserve((size_t)nover * k);
  h->c_dist.reserve((size_t)nover * k);
  h->c_len.reserve(nover);
  h->c_bound.reserve(np);
  gather_queries_kernel<<<nover, 128, 0, s>>>(d_q, h->c_idx.p, h->dim, h->c_q.p);
  gather_bound_kernel<<<grid1d(np, 256), 256, 0, s>>>(h->g_bound.p, h->c_idx.p, nover, np, h->c_bound.p);
  PXC_CUDA(cudaMemsetAsync(h->q_bad.p, 0, sizeof(int), s));
  prep_queries_u8_kernel<<<np, 128, 0, s>>>(h->c_q.p, nover, h->dim, h->dp, h->q_u8.p, h->q_norm.p, h->q_bad.p);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 3;
  group_launches(h, op, h->c_q.p, nover, k, h->c_bound.p, d_bitmap, h->c_ids.p, h->c_dist.p, h->c_len.p, s);
  h->last_redo += nover;
  scatter_results_kernel<<<nover, 128, 0, s>>>(h->c_ids.p, h->c_dist.p, h->c_len.p, h->c_idx.p, k, d_ids, d_dist,
                                               d_len);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 1;
}

// The K2 operand of the current mirror: centre, ranges, scale, f16 rows and
// row terms. Leaves k2_state = 2 when the store does not suit the screen
// (dim > 128, manhattan, or magnitudes whose squares leave the f32 range).
void build_k2(pxc_flat* h, cudaStream_t s) {
  h->k2_state = 2;
  const uint64_t n = h->nrank;
  const uint32_t dim = h->dim;
  if (n == 0 || dim > K2_MAX_DIM || h->metric == PXC_MANHATTAN) return;
  h->k2_mu.reserve(dim);
  h->k2_part.reserve((size_t)K2_MEAN_CHUNKS * dim);
  column_partial_kernel<<<dim3((dim + 31) / 32, K2_MEAN_CHUNKS), dim3(32, 8), 0, s>>>(h->rank_rows.p, n, dim,
                                                                                      h->k2_part.p);
  column_mean_kernel<<<(dim + 127) / 128, 128, 0, s>>>(h->k2_part.p, K2_MEAN_CHUNKS, dim, n, h->k2_mu.p);
  h->k2_dp = (dim + 63) / 64 * 64;
  h->k2_nrank_pad = (n + flat_tc::BN - 1) / flat_tc::BN * flat_tc::BN;
  h->k2_h.reserve(h->k2_nrank_pad);
  h->k2_stats.reserve(4);
  PXC_CUDA(cudaMemsetAsync(h->k2_stats.p, 0, 4 * sizeof(uint32_t), s));
  k2_row_stats_kernel<<<(unsigned)n, 128, 0, s>>>(h->rank_rows.p, n, dim, h->k2_mu.p, h->metric, h->k2_h.p,
                                                 h->k2_stats.p);
  PXC_CUDA(cudaGetLastError());
  uint32_t st[4];
  PXC_CUDA(cudaMemcpyAsync(st, h->k2_stats.p, sizeof(st), cudaMemcpyDeviceToHost, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  h->ctx->launches += 3;
  float f[4];
  std::memcpy(f, st, sizeof(f));
  for (float v : f)
    if (!std::isfinite(v) || v > 1e30f) return;
  if ((double)f[1] * f[1] > 1e36 || (double)f[2] * f[2] > 1e36) return;
  h->k2_ax = f[0] > 0.0f ? 14 - std::ilogb(f[0]) : 0;
  h->k2_op.reserve(h->k2_nrank_pad * h->k2_dp);
  k2_operand_kernel<<<(unsigned)h->k2_nrank_pad, 128, 0, s>>>(h->rank_rows.p, n, dim, h->k2_dp, h->k2_mu.p,
                                                             h->k2_ax, h->k2_op.p, h->k2_h.p);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 1;
  make_tmap_u8_2d(&h->k2_tmap_x, h->k2_op.p, (uint64_t)h->k2_dp * 2, h->k2_nrank_pad, flat_tc::KB_BYTES,
                  flat_tc::BN);
  PXC_CUDA(cudaStreamSynchronize(s));
  h->k2_state = 1;
}

// Searches K2 serves: no filter (the screen's operand is the whole mirror),
// k small enough for the over-fetch to carry a proof, a metric with a
// product form, and a store that fits the f16 operand.
bool k2_applicable(const pxc_flat* h, uint32_t k, const uint64_t* d_bitmap) {
  return d_bitmap == nullptr && k >= 1 && k <= K2_MAX_K && h->metric != PXC_MANHATTAN && h->dim <= K2_MAX_DIM &&
         h->nrank > 0;
}

// K2: the f16 screen (flat_scan_kernel<K2_KT, F16Scan>), the exact re-rank
// with its per-query proof, and for the queries left unproven an exact range
// scan (K1g for the few whose range overflows).
void search_k2(pxc_flat* h, const float* d_q, uint32_t nq, uint32_t k, uint64_t* d_ids, float* d_dist,
               uint32_t* d_len, cudaStream_t s) {
  const uint32_t nq_pad = (nq + flat_tc::BM - 1) / flat_tc::BM * flat_tc::BM;
  const uint32_t nqt = nq_pad / flat_tc::BM;
  const uint32_t dp = h->k2_dp;
  h->k2_q.reserve((size_t)nq_pad * dp);
  h->k2_meta.reserve(nq_pad);
  h->k2_coef.reserve(2 * (size_t)nq_pad);  // c_q, then delta_q
  k2_prep_queries_kernel<<<nq_pad, 128, 0, s>>>(d_q, nq, h->dim, dp, h->k2_mu.p, h->metric, h->k2_ax,
                                                reinterpret_cast<const float*>(h->k2_stats.p), h->k2_q.p,
                                                h->k2_meta.p);
  PXC_CUDA(cudaGetLastError());
  copy_coef_kernel<<<grid1d(nq_pad, 256), 256, 0, s>>>(h->k2_meta.p, nq_pad, h->k2_coef.p,
                                                       h->k2_coef.p + nq_pad);
  const uint32_t ntiles = (uint32_t)(h->k2_nrank_pad / flat_tc::BN);
  const uint32_t nsplit_req = choose_splits(nqt, ntiles, h->ctx->sm_count, K2_KT);
  const uint32_t tps = (ntiles + nsplit_req - 1) / nsplit_req;
  const uint32_t nsplit = (ntiles + tps - 1) / tps;
  h->part.reserve((size_t)nq_pad * nsplit * K2_KT);
  h->bound.reserve(nq_pad);
  h->done.reserve(nqt + (size_t)nqt * nsplit);
  PXC_CUDA(cudaMemsetAsync(h->bound.p, 0xFF, nq_pad * sizeof(uint32_t), s));  // reads as "no bound yet"
  PXC_CUDA(cudaMemsetAsync(h->done.p, 0, nqt * sizeof(uint32_t), s));
  PXC_CUDA(cudaMemsetAsync(h->done.p + nqt, 0xFF, (size_t)nqt * nsplit * sizeof(uint32_t), s));
  flat_tc::Params p;
  p.norms = h->k2_h.p;
  p.qcoef = h->k2_coef.p;
  p.qdelta = h->k2_coef.p + nq_pad;
  p.bound = reinterpret_cast<uint32_t*>(h->bound.p);
  p.done_count = h->done.p;
  p.done_list = h->done.p + nqt;
  p.out_part = h->part.p;
  p.status = h->d_status;
  p.nq = nq;
  p.k = k;  // the shared bound is min(last entry, k-th + delta_q): F16Scan::publish
  p.kblocks = dp * 2 / flat_tc::KB_BYTES;
  p.ntiles = ntiles;
  p.tiles_per_split = tps;
  p.nsplit = nsplit;
  p.stages = flat_tc::pick_stages<flat_tc::F16Scan>(p.kblocks);
  p.wait_ns = (uint64_t)h->ctx->wait_ms * 1000000ull;
  CUtensorMap tmap_q;
  make_tmap_u8_2d(&tmap_q, h->k2_q.p, (uint64_t)dp * 2, nq_pad, flat_tc::KB_BYTES, flat_tc::BM);
  const size_t smem = flat_tc::smem_bytes<flat_tc::F16Scan>(p.kblocks, p.stages);
  {
    ScanTimer timer(h, s);
    launch_tc<K2_KT, flat_tc::F16Scan>(tmap_q, h->k2_tmap_x, p, dim3(nqt, nsplit), smem, s);
    PXC_CUDA(cudaGetLastError());
    timer.stop();
  }
  uint32_t cap = 32;
  while (cap < nsplit * K2_KT) cap <<= 1;
  h->g_redo.reserve(nq);
  h->g_redo_idx.reserve(nq);
  h->g_redo_len.reserve(1);
  h->k2_kth.reserve(nq);
  k2_rerank_kernel<<<nq, 128, cap * sizeof(uint64_t), s>>>(h->part.p, nsplit, cap,
                                                           reinterpret_cast<const uint32_t*>(h->bound.p),
                                                           h->k2_meta.p, d_q, h->dim,
                                                           h->metric, h->rank_rows.p, h->rank_id.p,
                                                           (uint32_t)h->nrank, k, d_ids, d_dist, d_len, h->g_redo.p,
                                                           h->k2_kth.p);
  PXC_CUDA(cudaGetLastError());
  h->ctx->launches += 4;
  check_status_word(h->d_status, h->h_status, s, "flat search (tensor-core screen)");
  // the unproven queries: the exact range scan, then (on overflow) K1g
  size_t tb = 0;
  thrust::counting_iterator<uint32_t> it(0);
  PXC_CUDA(cub::DeviceSelect::Flagged(nullptr, tb, it, h->g_redo.p, h->g_redo_idx.p, h->g_redo_len.p, (int64_t)nq, s));
  h->tmp.reserve(std::max<size_t>(tb, 1));
  PXC_CUDA(cub::DeviceSelect::Flagged(h->tmp.p, tb, it, h->g_redo.p, h->g_redo_idx.p, h->g_redo_len.p, (int64_t)nq, s));
  PXC_CUDA(cudaMemcpyAsync(h->h_flag, h->g_redo_len.p, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
  PXC_CUDA(cudaStreamSynchronize(s));
  const uint32_t nredo = static_cast<uint32_t>(*h->h_flag);
  h->last_redo = nredo;
  h->ctx->launches += 2;
  if (nredo == 0) return;
  for (uint32_t b = 0; b < nredo; b += K2_RANGE_BATCH) {
    const uint32_t nb = std::min(K2_RANGE_BATCH, nredo - b);
    const uint32_t* idx = h->g_redo_idx.p + b;
    h->g_redo_q.reserve((size_t)nb * h->dim);
    h->k2_thr.reserve(nb);
    h->k2_range.reserve((size_t)nb * K2_RANGE_CAP);
    h->k2_range_cnt.reserve(nb);
    h->k2_ovf.reserve(nb);
    gather_queries_kernel<<<nb, 128, 0, s>>>(d_q, idx, h->dim, h->g_redo_q.p);
    gather_f32_kernel<<<grid1d(nb, 256), 256, 0, s>>>(h->k2_kth.p, idx, nb, h->k2_thr.p);
    PXC_CUDA(cudaMemsetAsync(h->k2_range_cnt.p, 0, nb * sizeof(uint32_t), s));
    k2_range_kernel<<<dim3(grid1d(h->nrank, 128), (nb + K2_RANGE_Q - 1) / K2_RANGE_Q), 128, 0, s>>>(
        h->g_redo_q.p, h->k2_thr.p, nb, h->rank_rows.p, (uint32_t)h->nrank, h->dim, h->metric, h->k2_range.p,
        h->k2_range_cnt.p);
    PXC_CUDA(cudaFuncSetAttribute(k2_range_finish_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)(K2_RANGE_CAP * sizeof(uint64_t))));
    k2_range_finish_kernel<<<nb, 256, K2_RANGE_CAP * sizeof(uint64_t), s>>>(
        h->k2_range.p, h->k2_range_cnt.p, idx, k, h->rank_id.p, d_ids, d_dist, d_len, h->k2_ovf.p);
    PXC_CUDA(cudaGetLastError());
    h->ctx->launches += 4;
    // overflowing queries (ties or near-ties beyond the collection's capacity): K1g
    h->k2_ovf_idx.reserve(nb);
    h->k2_ovf_len.reserve(1);
    tb = 0;
    PXC_CUDA(cub::DeviceSelect::Flagged(nullptr, tb, idx, h->k2_ovf.p, h->k2_ovf_idx.p, h->k2_ovf_len.p, (int64_t)nb, s));
    h->tmp.reserve(std::max<size_t>(tb, 1));
    PXC_CUDA(cub::DeviceSelect::Flagged(h->tmp.p, tb, idx, h->k2_ovf.p, h->k2_ovf_idx.p, h->k2_ovf_len.p, (int64_t)nb, s));
    PXC_CUDA(cudaMemcpyAsync(h->h_flag, h->k2_ovf_len.p, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    const uint32_t novf = static_cast<uint32_t>(*h->h_flag);
    h->ctx->launches += 2;
    if (novf == 0) continue;
    h->g_redo_q.reserve((size_t)novf * h->dim);
    h->g_redo_ids.reserve((size_t)novf * k);
    h->g_redo_dist.reserve((size_t)novf * k);
    h->g_redo_len.reserve(novf);
    gather_queries_kernel<<<novf, 128, 0, s>>>(d_q, h->k2_ovf_idx.p, h->dim, h->g_redo_q.p);
    PXC_CUDA(cudaGetLastError());
    search_generic(h, h->g_redo_q.p, novf, k, nullptr, h->g_redo_ids.p, h->g_redo_dist.p, h->g_redo_len.p, s);
    scatter_results_kernel<<<novf, 128, 0, s>>>(h->g_redo_ids.p, h->g_redo_dist.p, h->g_redo_len.p,
                                                h->k2_ovf_idx.p, k, d_ids, d_dist, d_len);
    PXC_CUDA(cudaGetLastError());
    h->ctx->launches += 2;
  }
}

void search_device(pxc_flat* h, const float* d_q, uint32_t nq, uint32_t k, const uint64_t* d_bitmap,
                   uint64_t* d_ids, float* d_dist, uint32_t* d_len, cudaStream_t s) {
  PXC_CONFIG(k <= PXC_MAX_K, "k", k, "exceeds the 16777216 result ceiling");
  h->last_redo = 0;
  if (h->dirty) rebuild_mirror(h, s);
  if (nq == 0) return;
  if (k == 0 || h->nrank == 0) {
    PXC_CUDA(cudaMemsetAsync(d_len, 0, nq * sizeof(uint32_t), s));
    return;
  }
  bool tc = h->all_u8 && h->metric == PXC_EUCLIDEAN && k <= GROUPED_MAX_K &&
            h->dim <= (uint32_t)flat_tc::MAX_KBLOCKS * flat_tc::KB_BYTES && h->nrank_pad > 0;
  if (tc) {
    const uint32_t nq_pad = (nq + flat_tc::BM - 1) / flat_tc::BM * flat_tc::BM;
    h->q_u8.reserve((size_t)nq_pad * h->dp);
    h->q_norm.reserve(nq_pad);
    h->q_bad.reserve(1);
    PXC_CUDA(cudaMemsetAsync(h->q_bad.p, 0, sizeof(int), s));
    prep_queries_u8_kernel<<<nq_pad, 128, 0, s>>>(d_q, nq, h->dim, h->dp, h->q_u8.p, h->q_norm.p, h->q_bad.p);
    PXC_CUDA(cudaGetLastError());
    h->ctx->launches += 1;
    PXC_CUDA(cudaMemcpyAsync(h->h_flag, h->q_bad.p, sizeof(int), cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    tc = (*h->h_flag == 0);
  }
  if (tc) {
    TcOperand op{&h->tmap_x, h->op_norm.p, h->nrank_pad, h->rank_id.p, h->nrank, h->op_u8.p};
    CUtensorMap tmap_f;
    if (d_bitmap) {
      // the filter's accepted ranks, compacted in rank order, as K1's database
      h->f_flags.reserve(h->nrank);
      h->f_acc.reserve(h->nrank);
      h->f_count.reserve(1);
      rank_flags_kernel<<<grid1d(h->nrank, 256), 256, 0, s>>>(h->rank_slot.p, h->nrank, d_bitmap, h->f_flags.p);
      size_t tb = 0;
      thrust::counting_iterator<uint32_t> it(0);
      PXC_CUDA(cub::DeviceSelect::Flagged(nullptr, tb, it, h->f_flags.p, h->f_acc.p, h->f_count.p, (int64_t)h->nrank, s));
      h->tmp.reserve(std::max<size_t>(tb, 1));
      PXC_CUDA(cub::DeviceSelect::Flagged(h->tmp.p, tb, it, h->f_flags.p, h->f_acc.p, h->f_count.p, (int64_t)h->nrank, s));
      PXC_CUDA(cudaMemcpyAsync(h->h_flag, h->f_count.p, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
      PXC_CUDA(cudaStreamSynchronize(s));
      const uint64_t nacc = static_cast<uint32_t>(*h->h_flag);
      h->ctx->launches += 3;
      if (nacc == 0) {
        PXC_CUDA(cudaMemsetAsync(d_len, 0, nq * sizeof(uint32_t), s));
        return;
      }
      const uint64_t npad = (nacc + flat_tc::BN - 1) / flat_tc::BN * flat_tc::BN;
      h->f_op.reserve(npad * h->dp);
      h->f_norm.reserve(npad);
      h->f_id.reserve(npad);
      gather_operand_kernel<<<(unsigned)npad, 64, 0, s>>>(h->op_u8.p, h->op_norm.p, h->rank_id.p, h->f_acc.p, nacc,
                                                         h->dp, h->f_op.p, h->f_norm.p, h->f_id.p);
      PXC_CUDA(cudaGetLastError());
      h->ctx->launches += 1;
      make_tmap_u8_2d(&tmap_f, h->f_op.p, h->dp, npad, flat_tc::KB_BYTES, flat_tc::BN);
      op = TcOperand{&tmap_f, h->f_norm.p, npad, h->f_id.p, nacc, h->f_op.p};
    }
    if (k <= TC_MAX_K)
      search_tc(h, op, d_q, nq, k, d_ids, d_dist, d_len, s);
    else
      search_tc_grouped(h, op, d_q, nq, k, d_bitmap, d_ids, d_dist, d_len, s);
    check_status_word(h->d_status, h->h_status, s, "flat search (tensor-core scan)");
    return;
  }
  if (k2_applicable(h, k, d_bitmap)) {
    if (h->k2_state == 0) build_k2(h, s);
    if (h->k2_state == 1) {
      search_k2(h, d_q, nq, k, d_ids, d_dist, d_len, s);
      return;
    }
  }
  search_generic(h, d_q, nq, k, d_bitmap, d_ids, d_dist, d_len, s);
}

}  // namespace

extern "C" {

pxc_status pxc_flat_create(pxc_ctx* ctx, uint32_t dim, int32_t metric, pxc_flat** out, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(out != nullptr, "out", 0, "output handle pointer is null");
    PXC_CONFIG(dim >= 1, "dim", dim, "must be at least 1; a 0-dimensional space makes all distances equal");
    PXC_CONFIG(dim <= (1u << 20), "dim", dim, "exceeds the 1048576 dimension ceiling");
    PXC_CONFIG(metric >= 0 && metric <= 3, "metric", metric, "unknown metric code");
    DeviceGuard g(ctx->device);
    pxc_flat* h = new (std::nothrow) pxc_flat();
    if (!h) throw make_failure(PXC_INTERNAL, 0, 0, nullptr, "out of host memory");
    h->ctx = ctx;
    h->dim = dim;
    h->metric = metric;
    cudaError_t e = cudaMallocHost(&h->h_flag, sizeof(int));
    if (e == cudaSuccess) e = cudaMallocHost(&h->h_status, 2 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMalloc(&h->d_status, 2 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(h->d_status, 0, 2 * sizeof(uint32_t));
    if (e != cudaSuccess) {
      pxc_flat_destroy(h);
      PXC_CUDA(e);
    }
    *out = h;
  });
}

void pxc_flat_destroy(pxc_flat* h) {
  if (!h) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(h->ctx->device);
  cudaStreamSynchronize(h->ctx->stream);
  if (h->ev_done) {
    cudaEventSynchronize(h->ev_done);  // a search on another stream may still be running
    cudaEventDestroy(h->ev_done);
  }
  if (h->ev_begin) cudaEventDestroy(h->ev_begin);
  if (h->ev_end) cudaEventDestroy(h->ev_end);
  if (h->h_flag) cudaFreeHost(h->h_flag);
  if (h->h_status) cudaFreeHost(h->h_status);
  if (h->d_status) cudaFree(h->d_status);
  delete h;
  if (prev >= 0) cudaSetDevice(prev);
}

pxc_status pxc_flat_sync(pxc_flat* h, const float* rows, const uint64_t* ids, const uint8_t* live,
                         uint64_t slot_begin, uint64_t nslots, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "handle", 0, "null flat handle");
    if (nslots == 0) return;
    PXC_CONFIG(rows != nullptr, "rows", 0, "null rows");
    PXC_CONFIG(slot_begin <= h->nslots, "slot_begin", slot_begin, "leaves a gap after the mirror's last slot");
    PXC_CONFIG(slot_begin + nslots < (1ull << 32), "slots", slot_begin + nslots, "the device mirror addresses at most 2^32 slots");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = h->ctx->stream;
    handoff_drain(h);
    const uint64_t dim = h->dim;
    // stage + validate before touching the mirror
    h->stage_f.reserve(nslots * dim);
    h->bad_idx.reserve(1);
    DBuf<uint8_t> flags;
    flags.reserve(nslots);
    PXC_CUDA(cudaMemcpyAsync(h->stage_f.p, rows, nslots * dim * sizeof(float), cudaMemcpyHostToDevice, s));
    PXC_CUDA(cudaMemsetAsync(h->bad_idx.p, 0xFF, sizeof(unsigned long long), s));
    validate_rows_kernel<<<(unsigned)nslots, 128, 0, s>>>(h->stage_f.p, nslots, h->dim, h->bad_idx.p, flags.p);
    PXC_CUDA(cudaGetLastError());
    unsigned long long bad = 0;
    PXC_CUDA(cudaMemcpyAsync(&bad, h->bad_idx.p, sizeof(bad), cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    if (bad != ~0ull)
      throw make_failure(PXC_NON_FINITE, bad, 0, nullptr, "vector component %llu is not finite", bad);
    ensure_capacity(h, slot_begin + nslots, s);
    PXC_CUDA(cudaMemcpyAsync(h->rows.p + slot_begin * dim, h->stage_f.p, nslots * dim * sizeof(float), cudaMemcpyDeviceToDevice, s));
    PXC_CUDA(cudaMemcpyAsync(h->rowflag.p + slot_begin, flags.p, nslots, cudaMemcpyDeviceToDevice, s));
    if (ids) {
      PXC_CUDA(cudaMemcpyAsync(h->ids.p + slot_begin, ids, nslots * sizeof(uint64_t), cudaMemcpyHostToDevice, s));
    } else {
      iota_ids_kernel<<<grid1d(nslots, 256), 256, 0, s>>>(h->ids.p + slot_begin, slot_begin, nslots);
    }
    if (live) {
      PXC_CUDA(cudaMemcpyAsync(h->live.p + slot_begin, live, nslots, cudaMemcpyHostToDevice, s));
    } else {
      PXC_CUDA(cudaMemsetAsync(h->live.p + slot_begin, 1, nslots, s));
    }
    PXC_CUDA(cudaStreamSynchronize(s));
    h->nslots = std::max(h->nslots, slot_begin + nslots);
    h->dirty = true;
  });
}

pxc_status pxc_flat_truncate(pxc_flat* h, uint64_t nslots, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "handle", 0, "null flat handle");
    std::lock_guard<std::mutex> lock(h->mu);
    PXC_CONFIG(nslots <= h->nslots, "nslots", nslots, "truncate cannot grow the mirror");
    DeviceGuard g(h->ctx->device);
    handoff_drain(h);  // the next search rebuilds the mirror that earlier searches may still read
    h->nslots = nslots;
    h->dirty = true;
  });
}

uint64_t pxc_flat_len(const pxc_flat* h) {
  if (!h) return 0;
  pxc_flat* m = const_cast<pxc_flat*>(h);
  std::lock_guard<std::mutex> lock(m->mu);
  if (m->dirty) {
    try {
      DeviceGuard g(m->ctx->device);
      rebuild_mirror(m, m->ctx->stream);
    } catch (...) {
      return 0;
    }
  }
  return m->nrank;
}

float pxc_flat_last_scan_ms(pxc_flat* h) {
  if (!h || !h->ev_recorded) return -1.0f;
  float ms = -1.0f;
  if (cudaEventSynchronize(h->ev_end) != cudaSuccess) return -1.0f;
  if (cudaEventElapsedTime(&ms, h->ev_begin, h->ev_end) != cudaSuccess) return -1.0f;
  return ms;
}

uint32_t pxc_flat_last_redone(const pxc_flat* h) { return h ? h->last_redo : 0u; }

int32_t pxc_flat_path(const pxc_flat* h) {
  if (!h) return -1;
  pxc_flat* m = const_cast<pxc_flat*>(h);
  std::lock_guard<std::mutex> lock(m->mu);
  if (m->dirty) {
    try {
      DeviceGuard g(m->ctx->device);
      rebuild_mirror(m, m->ctx->stream);
    } catch (...) {
      return -1;
    }
  }
  if (m->all_u8 && m->metric == PXC_EUCLIDEAN && m->dim <= (uint32_t)flat_tc::MAX_KBLOCKS * flat_tc::KB_BYTES &&
      m->nrank > 0)
    return 1;
  if (!k2_applicable(m, 1, nullptr)) return 0;
  if (m->k2_state == 0) {
    try {
      DeviceGuard g(m->ctx->device);
      handoff_drain(m);
      build_k2(m, m->ctx->stream);
    } catch (...) {
      return -1;
    }
  }
  return m->k2_state == 1 ? 2 : 0;
}

pxc_status pxc_flat_search_device(pxc_flat* h, const float* d_queries, uint32_t nq, uint32_t k,
                                  const uint64_t* d_bitmap, uint64_t* d_out_ids, float* d_out_dist,
                                  uint32_t* d_out_len, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "handle", 0, "null flat handle");
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->ctx->stream;
    handoff_wait(h, s);
    search_device(h, d_queries, nq, k, d_bitmap, d_out_ids, d_out_dist, d_out_len, s);
    handoff_done(h, s);
  });
}

pxc_status pxc_flat_search_sharded(pxc_flat* h, const float* d_queries, uint32_t nq, uint32_t k,
                                   const uint64_t* d_bitmap, uint64_t* d_out_ids, float* d_out_dist,
                                   uint32_t* d_out_len, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "handle", 0, "null flat handle");
    PXC_CONFIG(k <= PXC_MAX_K, "k", k, "exceeds the 16777216 result ceiling");
    pxc_ctx* ctx = h->ctx;
    PXC_CONFIG((uint64_t)ctx->nranks * k <= 8192, "nranks*k", (uint64_t)ctx->nranks * k,
               "the merge holds at most 8192 candidates per query");
    if (nq == 0) return;
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    std::lock_guard<std::mutex> comm_lock(ctx->comm_mu);
    // the local search writes straight into this rank's exchange segment
    unsigned char* send = exchange_send_buffer(ctx, exchange_segment_bytes(nq, k));
    const size_t n = (size_t)nq * k;
    handoff_wait(h, s);
    search_device(h, d_queries, nq, k, d_bitmap, reinterpret_cast<uint64_t*>(send),
                  reinterpret_cast<float*>(send + n * 8), reinterpret_cast<uint32_t*>(send + n * 12), s);
    exchange_and_merge(ctx, send, nq, k, k, d_out_ids, d_out_dist, d_out_len, s);
    handoff_done(h, s);
  });
}

pxc_status pxc_flat_search_sharded_owned(pxc_flat* h, const float* d_queries, uint32_t nq, uint32_t k,
                                         const uint64_t* d_bitmap, uint64_t* d_out_ids, float* d_out_dist,
                                         uint32_t* d_out_len, void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "handle", 0, "null flat handle");
    PXC_CONFIG(k <= PXC_MAX_K, "k", k, "exceeds the 16777216 result ceiling");
    pxc_ctx* ctx = h->ctx;
    PXC_CONFIG((uint64_t)ctx->nranks * k <= 8192, "nranks*k", (uint64_t)ctx->nranks * k,
               "the merge holds at most 8192 candidates per query");
    if (nq == 0) return;
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    std::lock_guard<std::mutex> comm_lock(ctx->comm_mu);
    handoff_wait(h, s);
    if (ctx->nranks <= 1 || ctx->comm == nullptr) {  // one rank owns every query
      search_device(h, d_queries, nq, k, d_bitmap, d_out_ids, d_out_dist, d_out_len, s);
    } else {
      unsigned char* send = exchange_send_buffer(ctx, exchange_segment_bytes(nq, k));
      const size_t n = (size_t)nq * k;
      uint64_t* ids = reinterpret_cast<uint64_t*>(send);
      float* dist = reinterpret_cast<float*>(send + n * 8);
      uint32_t* lens = reinterpret_cast<uint32_t*>(send + n * 12);
      search_device(h, d_queries, nq, k, d_bitmap, ids, dist, lens, s);
      exchange_to_owners(ctx, ids, dist, lens, nq, k, k, d_out_ids, d_out_dist, d_out_len, s);
    }
    handoff_done(h, s);
  });
}

}  // extern "C"

namespace {
// The host-buffer search, with the filter given as a HOST bitmap, or as
// conditions evaluated on the device into the bitmap (where != nullptr).
struct Where {
  pxc_columns* cols;
  const pxc_condition* conds;
  uint32_t ncond;
  const pxc_operand* ops;
  uint32_t nops;
};
void flat_search_host(pxc_flat* h, const float* queries, uint32_t nq, uint32_t k, const uint64_t* bitmap,
                      const Where* where, uint64_t* out_ids, float* out_dist, uint32_t* out_len);
}  // namespace

extern "C" {

pxc_status pxc_flat_search_where(pxc_flat* h, pxc_columns* cols, const pxc_condition* conds, uint32_t ncond,
                                 const pxc_operand* operands, uint32_t noperands, const float* queries, uint32_t nq,
                                 uint32_t k, uint64_t* out_ids, float* out_dist, uint32_t* out_len, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr && cols != nullptr, "handle", 0, "null handle");
    PXC_CONFIG(k <= PXC_MAX_K, "k", k, "exceeds the 16777216 result ceiling");
    if (nq == 0) return;
    const Where w{cols, conds, ncond, operands, noperands};
    flat_search_host(h, queries, nq, k, nullptr, &w, out_ids, out_dist, out_len);
  });
}

pxc_status pxc_flat_search(pxc_flat* h, const float* queries, uint32_t nq, uint32_t k,
                           const uint64_t* bitmap, uint64_t* out_ids, float* out_dist,
                           uint32_t* out_len, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "handle", 0, "null flat handle");
    PXC_CONFIG(k <= PXC_MAX_K, "k", k, "exceeds the 16777216 result ceiling");
    if (nq == 0) return;
    flat_search_host(h, queries, nq, k, bitmap, nullptr, out_ids, out_dist, out_len);
  });
}

}  // extern "C"

namespace {
void flat_search_host(pxc_flat* h, const float* queries, uint32_t nq, uint32_t k, const uint64_t* bitmap,
                      const Where* where, uint64_t* out_ids, float* out_dist, uint32_t* out_len) {
  {
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = h->ctx->stream;
    handoff_wait(h, s);
    const uint64_t dim = h->dim;
    DBuf<float>& dq = h->io_q;
    DBuf<uint64_t>& dbm = h->io_bm;
    DBuf<uint64_t>& dids = h->io_ids;
    DBuf<float>& ddist = h->io_dist;
    DBuf<uint32_t>& dlen = h->io_len;
    dq.reserve((size_t)nq * dim);
    dlen.reserve(nq);
    if (k > 0) {
      dids.reserve((size_t)nq * k);
      ddist.reserve((size_t)nq * k);
    }
    PXC_CUDA(cudaMemcpyAsync(dq.p, queries, (size_t)nq * dim * sizeof(float), cudaMemcpyHostToDevice, s));
    const bool filtered = bitmap != nullptr || where != nullptr;
    if (filtered) {
      if (h->dirty) rebuild_mirror(h, s);
      uint64_t words = (h->nslots + 63) / 64;
      dbm.reserve(std::max<uint64_t>(words, 1));
      if (words && bitmap)
        PXC_CUDA(cudaMemcpyAsync(dbm.p, bitmap, words * sizeof(uint64_t), cudaMemcpyHostToDevice, s));
      if (words && where) {
        pxc_error e{};
        if (pxc_columns_eval(where->cols, h->nslots, where->conds, where->ncond, where->ops, where->nops, dbm.p, s,
                             &e) != PXC_OK)
          throw make_failure((pxc_status)e.code, e.a, e.b, e.parameter, "%s", e.detail);
      }
    }
    search_device(h, dq.p, nq, k, filtered ? dbm.p : nullptr, dids.p, ddist.p, dlen.p, s);
    if (k > 0) {
      PXC_CUDA(cudaMemcpyAsync(out_ids, dids.p, (size_t)nq * k * sizeof(uint64_t), cudaMemcpyDeviceToHost, s));
      PXC_CUDA(cudaMemcpyAsync(out_dist, ddist.p, (size_t)nq * k * sizeof(float), cudaMemcpyDeviceToHost, s));
    }
    PXC_CUDA(cudaMemcpyAsync(out_len, dlen.p, nq * sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    handoff_done(h, s);
    PXC_CUDA(cudaStreamSynchronize(s));
  }
}
}  // namespace

// ---------------------------------------------------------------------------
// Allocation-free flat search (no counterpart in the reference).
//
// For callers that cannot allocate device memory: a host runtime that has
// reserved the whole device for its own pool (cudaMalloc would fail), or a
// latency-bound serving loop that cannot afford the implicit device-wide
// synchronisation of cudaMalloc/cudaFree. It runs the tensor-core scan (K1)
// with every per-call scratch buffer carved out of one file-scope device
// array, so the call allocates nothing: no cudaMalloc, no cudaFree, no
// allocating library routine.
//
// Limits: at most NOALLOC_MAX_QUERIES queries per call, k <= 16, dim <= 256,
// an integer euclidean store (the K1 conditions), and a device mirror that is
// already built (call pxc_flat_len or any search once after pxc_flat_sync;
// building the mirror allocates). The array costs NOALLOC_BYTES of device
// memory on every GPU that loads the library, until the process exits.
//
// The array is shared by every call and keeps the last call's contents; the
// parts that must start from a known value are reset by each call. Calls whose
// GPU work overlaps would race on it: within a process this entry point
// serialises its calls and returns only after its work has finished.
//
// Set-up: the first call on a device looks up the array's device address with
// cudaGetSymbolAddress (with that device current). Every call synchronises
// its stream (after the query check and at the end), so it returns with its
// work finished.
// ---------------------------------------------------------------------------
namespace {
constexpr uint32_t NOALLOC_MAX_QUERIES = 2048;
constexpr uint32_t NOALLOC_MAX_SPLITS = 32;
constexpr uint32_t NOALLOC_MAX_KT = 16;
constexpr uint32_t NOALLOC_MAX_DIM = 256;
constexpr size_t NOALLOC_Q_OFF = 0;
constexpr size_t NOALLOC_PART_OFF = NOALLOC_Q_OFF + (size_t)NOALLOC_MAX_QUERIES * NOALLOC_MAX_DIM;
constexpr size_t NOALLOC_NORM_OFF =
    NOALLOC_PART_OFF + (size_t)NOALLOC_MAX_QUERIES * NOALLOC_MAX_SPLITS * NOALLOC_MAX_KT * sizeof(uint64_t);
constexpr size_t NOALLOC_BOUND_OFF = NOALLOC_NORM_OFF + (size_t)NOALLOC_MAX_QUERIES * sizeof(int32_t);
constexpr size_t NOALLOC_DONE_OFF = NOALLOC_BOUND_OFF + (size_t)NOALLOC_MAX_QUERIES * sizeof(int32_t);
constexpr uint32_t NOALLOC_MAX_QTILES = NOALLOC_MAX_QUERIES / flat_tc::BM;
constexpr size_t NOALLOC_BAD_OFF =
    NOALLOC_DONE_OFF + ((size_t)NOALLOC_MAX_QTILES * (1 + NOALLOC_MAX_SPLITS) * sizeof(uint32_t) + 255) / 256 * 256;
constexpr size_t NOALLOC_BYTES = NOALLOC_BAD_OFF + 256;  // ~8.6 MiB
}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_BYTES];

namespace {
std::mutex g_noalloc_mu;        // serialises calls (they share the array)
void* g_noalloc_addr[256] = {};  // device address of the array, per device ordinal

unsigned char* noalloc_scratch(int device) {
  if (device < 0 || device >= 256)
    throw make_failure(PXC_CONFIGURATION, (uint64_t)device, 0, "device", "device ordinal out of range");
  if (!g_noalloc_addr[device]) {
    void* p = nullptr;
    PXC_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_addr[device] = p;
  }
  return static_cast<unsigned char*>(g_noalloc_addr[device]);
}
}  // namespace

extern "C" pxc_status pxc_flat_search_noalloc(pxc_flat* h, const float* d_queries, uint32_t nq, uint32_t k,
                                              uint64_t* d_out_ids, float* d_out_dist, uint32_t* d_out_len,
                                              void* stream, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "handle", 0, "null flat handle");
    if (nq > NOALLOC_MAX_QUERIES)
      throw make_failure(PXC_CAPACITY, NOALLOC_MAX_QUERIES, nq, nullptr,
                         "allocation-free search: at most %u queries per call", NOALLOC_MAX_QUERIES);
    PXC_CONFIG(k <= NOALLOC_MAX_KT, "k", k, "allocation-free search supports k <= 16");
    std::lock_guard<std::mutex> global(g_noalloc_mu);
    std::lock_guard<std::mutex> lock(h->mu);
    DeviceGuard g(h->ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->ctx->stream;
    PXC_CONFIG(!h->dirty, "mirror", 0,
               "the device mirror is not built; call pxc_flat_len or a search once after pxc_flat_sync");
    unsigned char* base = noalloc_scratch(h->ctx->device);
    if (nq == 0) return;
    if (k == 0 || h->nrank == 0) {
      PXC_CUDA(cudaMemsetAsync(d_out_len, 0, nq * sizeof(uint32_t), s));
      PXC_CUDA(cudaStreamSynchronize(s));
      return;
    }
    PXC_CONFIG(h->all_u8 && h->metric == PXC_EUCLIDEAN && h->dim <= NOALLOC_MAX_DIM && h->nrank_pad > 0, "store",
               0, "allocation-free search needs a euclidean store of integers in [0,255] with dim <= 256");
    uint8_t* q_u8 = base + NOALLOC_Q_OFF;
    uint64_t* part = reinterpret_cast<uint64_t*>(base + NOALLOC_PART_OFF);
    int32_t* q_norm = reinterpret_cast<int32_t*>(base + NOALLOC_NORM_OFF);
    int32_t* bound = reinterpret_cast<int32_t*>(base + NOALLOC_BOUND_OFF);
    uint32_t* done = reinterpret_cast<uint32_t*>(base + NOALLOC_DONE_OFF);
    int* q_bad = reinterpret_cast<int*>(base + NOALLOC_BAD_OFF);

    const uint32_t nq_pad = (nq + flat_tc::BM - 1) / flat_tc::BM * flat_tc::BM;
    PXC_CUDA(cudaMemsetAsync(q_bad, 0, sizeof(int), s));
    prep_queries_u8_kernel<<<nq_pad, 128, 0, s>>>(d_queries, nq, h->dim, h->dp, q_u8, q_norm, q_bad);
    PXC_CUDA(cudaGetLastError());
    PXC_CUDA(cudaMemcpyAsync(h->h_flag, q_bad, sizeof(int), cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    PXC_CONFIG(*h->h_flag == 0, "queries", 0,
               "allocation-free search needs query components that are integers in [0,255]");

    const uint32_t KT = k <= 1 ? 1 : k <= 4 ? 4 : k <= 10 ? 10 : 16;
    const uint32_t nqt = nq_pad / flat_tc::BM;
    const uint32_t ntiles = (uint32_t)(h->nrank_pad / flat_tc::BN);
    const uint32_t nsplit_req = std::min(choose_splits(nqt, ntiles, h->ctx->sm_count, KT), NOALLOC_MAX_SPLITS);
    const uint32_t tps = (ntiles + nsplit_req - 1) / nsplit_req;
    const uint32_t nsplit = (ntiles + tps - 1) / tps;
    // reset what must start from a known value
    PXC_CUDA(cudaMemsetAsync(bound, 0x3F, nq_pad * sizeof(int32_t), s));
    PXC_CUDA(cudaMemsetAsync(done, 0, nqt * sizeof(uint32_t), s));
    PXC_CUDA(cudaMemsetAsync(done + nqt, 0xFF, (size_t)nqt * nsplit * sizeof(uint32_t), s));
    flat_tc::Params p;
    p.norms = h->op_norm.p;
    p.qcoef = nullptr;
    p.qdelta = nullptr;
    p.bound = reinterpret_cast<uint32_t*>(bound);
    p.done_count = done;
    p.done_list = done + nqt;
    p.out_part = part;
    p.status = h->d_status;
    p.nq = nq;
    p.k = k;
    p.kblocks = h->dp / flat_tc::KB_BYTES;
    p.ntiles = ntiles;
    p.tiles_per_split = tps;
    p.nsplit = nsplit;
    p.stages = flat_tc::pick_stages<flat_tc::U8Scan>(p.kblocks);
    p.wait_ns = (uint64_t)h->ctx->wait_ms * 1000000ull;
    CUtensorMap tmap_q;
    make_tmap_u8_2d(&tmap_q, q_u8, h->dp, nq_pad, flat_tc::KB_BYTES, flat_tc::BM);
    const size_t smem = flat_tc::smem_bytes<flat_tc::U8Scan>(p.kblocks, p.stages);
    const dim3 grid(nqt, nsplit);
    switch (KT) {
      case 1: launch_tc<1>(tmap_q, h->tmap_x, p, grid, smem, s); break;
      case 4: launch_tc<4>(tmap_q, h->tmap_x, p, grid, smem, s); break;
      case 10: launch_tc<10>(tmap_q, h->tmap_x, p, grid, smem, s); break;
      default: launch_tc<16>(tmap_q, h->tmap_x, p, grid, smem, s); break;
    }
    PXC_CUDA(cudaGetLastError());
    uint32_t cap = 32;
    while (cap < nsplit * KT) cap <<= 1;
    const size_t msmem = cap * sizeof(uint64_t);
    if (msmem > 48 * 1024)
      PXC_CUDA(cudaFuncSetAttribute(merge_u8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msmem));
    merge_u8_kernel<<<nq, 256, msmem, s>>>(part, nsplit, KT, cap, k, q_norm, h->rank_id.p, (uint32_t)h->nrank,
                                           d_out_ids, d_out_dist, d_out_len, nullptr);
    PXC_CUDA(cudaGetLastError());
    h->ctx->launches += 3;
    check_status_word(h->d_status, h->h_status, s, "allocation-free flat search");  // synchronises the stream
  });
}
