// pxo.cpp — CPU oracle (test infrastructure, never the product path).
//
// A C++17 restatement of the Rust reference's hot-path arithmetic. It must be
// compiled with -ffp-contract=off and without -ffast-math: rustc never
// contracts a*b+c into an FMA, and the reference has no mul_add, so IEEE
// single-precision operations in the same order reproduce its f32 results.
// Each function cites the reference file:line it restates.
#include "pxo.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <functional>
#include <queue>
#include <unordered_map>
#include <thread>
#include <vector>

namespace {

constexpr size_t LANES = 8;  // distance.rs:72

// distance.rs:534-538 — pairwise reduce of the eight lane accumulators.
inline float reduce8(const float* acc) {
  float a = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  float b = (acc[4] + acc[5]) + (acc[6] + acc[7]);
  return a + b;
}

// distance.rs:267-283
inline float l2_unrolled(const float* a, const float* b, size_t dim) {
  float acc[LANES] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t full = dim / LANES * LANES;
  for (size_t i = 0; i < full; i += LANES)
    for (size_t l = 0; l < LANES; ++l) {
      float d = a[i + l] - b[i + l];
      acc[l] += d * d;
    }
  float tail = 0.0f;
  for (size_t i = full; i < dim; ++i) {
    float d = a[i] - b[i];
    tail += d * d;
  }
  return reduce8(acc) + tail;
}

// distance.rs:317-331
inline float dot_unrolled(const float* a, const float* b, size_t dim) {
  float acc[LANES] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t full = dim / LANES * LANES;
  for (size_t i = 0; i < full; i += LANES)
    for (size_t l = 0; l < LANES; ++l) acc[l] += a[i + l] * b[i + l];
  float tail = 0.0f;
  for (size_t i = full; i < dim; ++i) tail += a[i] * b[i];
  return reduce8(acc) + tail;
}

// distance.rs manhattan_unrolled
inline float l1_unrolled(const float* a, const float* b, size_t dim) {
  float acc[LANES] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t full = dim / LANES * LANES;
  for (size_t i = 0; i < full; i += LANES)
    for (size_t l = 0; l < LANES; ++l) acc[l] += std::fabs(a[i + l] - b[i + l]);
  float tail = 0.0f;
  for (size_t i = full; i < dim; ++i) tail += std::fabs(a[i] - b[i]);
  return reduce8(acc) + tail;
}

// kmeans.rs:234-241 and product.rs:529-547 — one accumulator, in order.
inline float l2_sequential(const float* a, const float* b, size_t dim) {
  float sum = 0.0f;
  for (size_t i = 0; i < dim; ++i) {
    float d = a[i] - b[i];
    sum += d * d;
  }
  return sum;
}

// space.rs:148-156
inline float space_distance(int metric, const float* a, const float* b, size_t dim) {
  switch (metric) {
    case PXO_EUCLIDEAN: return l2_unrolled(a, b, dim);
    case PXO_COSINE: return 1.0f - dot_unrolled(a, b, dim);
    case PXO_INNER_PRODUCT: return -dot_unrolled(a, b, dim);
    default: return l1_unrolled(a, b, dim);
  }
}

// f32::total_cmp key (documented in the Rust std reference): flip the
// magnitude bits of negative numbers so the signed integer order is total.
inline int32_t total_key(float f) {
  int32_t b;
  std::memcpy(&b, &f, 4);
  return b ^ static_cast<int32_t>(static_cast<uint32_t>(b >> 31) >> 1);
}

struct Hit {
  float dist;
  uint64_t id;
};
// SearchResult's Ord (topk.rs:63-67): distance.total_cmp, then id.
inline bool hit_less(const Hit& a, const Hit& b) {
  int32_t ka = total_key(a.dist), kb = total_key(b.dist);
  if (ka != kb) return ka < kb;
  return a.id < b.id;
}

// TopK (topk.rs:93-191): bounded max-heap keeping the k smallest.
class TopK {
 public:
  explicit TopK(size_t k) : k_(k) { heap_.reserve(k + 1); }
  void push(uint64_t id, float d) {
    if (k_ == 0) return;
    Hit c{d, id};
    auto cmp = [](const Hit& a, const Hit& b) { return hit_less(a, b); };
    if (heap_.size() < k_) {
      heap_.push_back(c);
      std::push_heap(heap_.begin(), heap_.end(), cmp);
      return;
    }
    if (hit_less(c, heap_.front())) {
      std::pop_heap(heap_.begin(), heap_.end(), cmp);
      heap_.back() = c;
      std::push_heap(heap_.begin(), heap_.end(), cmp);
    }
  }
  std::vector<Hit> sorted() const {
    std::vector<Hit> v = heap_;
    std::sort(v.begin(), v.end(), hit_less);
    return v;
  }

 private:
  size_t k_;
  std::vector<Hit> heap_;
};

inline bool bit_set(const uint64_t* bitmap, uint64_t s) {
  return bitmap == nullptr || ((bitmap[s >> 6] >> (s & 63)) & 1u);
}

void parallel_for(uint64_t n, int threads, const std::function<void(uint64_t, uint64_t)>& fn) {
  if (threads <= 1 || n < 2) {
    fn(0, n);
    return;
  }
  uint64_t t = std::min<uint64_t>(threads, n);
  std::vector<std::thread> pool;
  for (uint64_t i = 0; i < t; ++i) {
    uint64_t b = n * i / t, e = n * (i + 1) / t;
    pool.emplace_back([&, b, e] { fn(b, e); });
  }
  for (auto& th : pool) th.join();
}

// ---------------------------------------------------------------------------
// rand restatement. ChaCha (D. J. Bernstein, "ChaCha, a variant of Salsa20")
// with 8 rounds, 64-bit block counter in words 12-13 and a 64-bit stream id
// in words 14-15 (zero for the generator), blocks emitted four at a time into
// a 64-word buffer; seed_from_u64 expands the u64 with PCG32 (XSH-RR, O'Neill
// 2014) into the 32-byte key; ranges follow rand 0.8's documented
// widening-multiply rejection (integers) and [1,2)-mantissa method (floats).
// The block function is pinned by RFC 8439's and the 8-round zero-key known
// answers (tests/test_rng_kat.py); the draws of the Rust crates themselves are
// not (no golden draw exists in the reference).
// ---------------------------------------------------------------------------
inline uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

void chacha_block(const uint32_t key[8], uint64_t counter, uint64_t stream, uint32_t out[16], int rounds) {
  uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                    key[0], key[1], key[2], key[3], key[4], key[5], key[6], key[7],
                    static_cast<uint32_t>(counter), static_cast<uint32_t>(counter >> 32),
                    static_cast<uint32_t>(stream), static_cast<uint32_t>(stream >> 32)};
  uint32_t x[16];
  std::memcpy(x, s, sizeof(x));
  auto qr = [&](int a, int b, int c, int d) {
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 16);
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 12);
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 8);
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 7);
  };
  for (int i = 0; i < rounds; i += 2) {
    qr(0, 4, 8, 12); qr(1, 5, 9, 13); qr(2, 6, 10, 14); qr(3, 7, 11, 15);
    qr(0, 5, 10, 15); qr(1, 6, 11, 12); qr(2, 7, 8, 13); qr(3, 4, 9, 14);
  }
  for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
}

void rng_refill(pxo_rng* r) {
  for (int b = 0; b < 4; ++b) chacha_block(r->key, r->counter + b, 0, r->buf + 16 * b, 8);
  r->counter += 4;
  r->index = 0;
}

}  // namespace

extern "C" {

void pxo_chacha_block(const uint32_t key[8], uint64_t counter, uint64_t stream, int rounds, uint32_t out[16]) {
  chacha_block(key, counter, stream, out, rounds);
}

float pxo_squared_euclidean(const float* a, const float* b, uint64_t dim) { return l2_unrolled(a, b, dim); }
float pxo_squared_euclidean_scalar(const float* a, const float* b, uint64_t dim) { return l2_sequential(a, b, dim); }
float pxo_dot(const float* a, const float* b, uint64_t dim) { return dot_unrolled(a, b, dim); }
float pxo_manhattan(const float* a, const float* b, uint64_t dim) { return l1_unrolled(a, b, dim); }
float pxo_cosine_normalized(const float* a, const float* b, uint64_t dim) { return 1.0f - dot_unrolled(a, b, dim); }

// distance.rs:cosine_unrolled — both norms on the fly; zero vector scores 1.0.
float pxo_cosine(const float* a, const float* b, uint64_t dim) {
  float ad[LANES] = {0}, aa[LANES] = {0}, ab[LANES] = {0};
  size_t full = dim / LANES * LANES;
  for (size_t i = 0; i < full; i += LANES)
    for (size_t l = 0; l < LANES; ++l) {
      float x = a[i + l], y = b[i + l];
      ad[l] += x * y;
      aa[l] += x * x;
      ab[l] += y * y;
    }
  float d = 0, na = 0, nb = 0;
  for (size_t i = full; i < dim; ++i) {
    d += a[i] * b[i];
    na += a[i] * a[i];
    nb += b[i] * b[i];
  }
  float dotv = reduce8(ad) + d, n1 = reduce8(aa) + na, n2 = reduce8(ab) + nb;
  float denom = std::sqrt(n1 * n2);
  if (denom <= 0.0f) return 1.0f;
  return 1.0f - dotv / denom;
}

// distance.rs:508-517 — n = sqrt(dot(v,v)); if 0<n<inf, v *= 1/n.
float pxo_normalize_in_place(float* v, uint64_t dim) {
  float n = std::sqrt(dot_unrolled(v, v, dim));
  if (n > 0.0f && std::isfinite(n)) {
    float inv = 1.0f / n;
    for (uint64_t i = 0; i < dim; ++i) v[i] *= inv;
  }
  return n;
}

float pxo_space_distance(int metric, const float* a, const float* b, uint64_t dim) {
  return space_distance(metric, a, b, dim);
}

// space.rs:104-120 (validate) and :130-138 (prepare)
int64_t pxo_prepare(int metric, float* rows, uint64_t n, uint64_t dim) {
  for (uint64_t i = 0; i < n * dim; ++i)
    if (!std::isfinite(rows[i])) return static_cast<int64_t>(i);
  if (metric == PXO_COSINE)
    for (uint64_t r = 0; r < n; ++r) pxo_normalize_in_place(rows + r * dim, dim);
  return -1;
}

// flat.rs:153-169 — scan live slots in slot order, filter, TopK.
void pxo_flat_search(const float* data, const uint64_t* ids, const uint8_t* live,
                     uint64_t nslots, uint64_t dim, int metric, const float* queries,
                     uint64_t nq, uint64_t k, const uint64_t* bitmap, uint64_t* out_ids,
                     float* out_dist, uint32_t* out_len, int threads) {
  parallel_for(nq, threads, [&](uint64_t qb, uint64_t qe) {
    for (uint64_t q = qb; q < qe; ++q) {
      TopK top(k);
      const float* qv = queries + q * dim;
      for (uint64_t s = 0; s < nslots; ++s) {
        if (live && !live[s]) continue;
        if (!bit_set(bitmap, s)) continue;
        top.push(ids ? ids[s] : s, space_distance(metric, qv, data + s * dim, dim));
      }
      auto v = top.sorted();
      for (size_t i = 0; i < v.size(); ++i) {
        out_ids[q * k + i] = v[i].id;
        out_dist[q * k + i] = v[i].dist;
      }
      out_len[q] = static_cast<uint32_t>(v.size());
    }
  });
}

// recall.rs:176-187
float pxo_recall_overlap(const uint64_t* exact, uint32_t exact_len, const uint64_t* approx,
                         uint32_t approx_len) {
  if (exact_len == 0) return 1.0f;
  uint32_t hits = 0;
  for (uint32_t i = 0; i < approx_len; ++i)
    for (uint32_t j = 0; j < exact_len; ++j)
      if (approx[i] == exact[j]) {
        ++hits;
        break;
      }
  return static_cast<float>(hits) / static_cast<float>(exact_len);
}

// ---- rand ----
void pxo_rng_seed_from_u64(pxo_rng* r, uint64_t state) {
  const uint64_t MUL = 6364136223846793005ull, INC = 11634580027462260723ull;
  for (int i = 0; i < 8; ++i) {
    state = state * MUL + INC;
    uint32_t xorshifted = static_cast<uint32_t>(((state >> 18) ^ state) >> 27);
    uint32_t rot = static_cast<uint32_t>(state >> 59);
    r->key[i] = (xorshifted >> rot) | (xorshifted << ((32 - rot) & 31));
  }
  r->counter = 0;
  r->index = 64;  // empty buffer: first draw refills
}

uint32_t pxo_rng_next_u32(pxo_rng* r) {
  if (r->index >= 64) rng_refill(r);
  return r->buf[r->index++];
}

uint64_t pxo_rng_next_u64(pxo_rng* r) {
  if (r->index < 63) {
    uint64_t lo = r->buf[r->index], hi = r->buf[r->index + 1];
    r->index += 2;
    return (hi << 32) | lo;
  }
  if (r->index >= 64) {
    rng_refill(r);
    uint64_t lo = r->buf[0], hi = r->buf[1];
    r->index = 2;
    return (hi << 32) | lo;
  }
  uint64_t lo = r->buf[63];
  rng_refill(r);
  uint64_t hi = r->buf[0];
  r->index = 1;
  return (hi << 32) | lo;
}

// Uniform integer in [0, n): widening multiply with a leading-zeros zone.
uint64_t pxo_rng_gen_range_usize(pxo_rng* r, uint64_t n) {
  uint64_t range = n;  // high - low, inclusive range = n-1 - 0 + 1
  if (range == 0) return pxo_rng_next_u64(r);
  uint64_t zone = (range << __builtin_clzll(range)) - 1;
  for (;;) {
    uint64_t v = pxo_rng_next_u64(r);
    unsigned __int128 m = static_cast<unsigned __int128>(v) * range;
    uint64_t hi = static_cast<uint64_t>(m >> 64), lo = static_cast<uint64_t>(m);
    if (lo <= zone) return hi;
  }
}

// Uniform f64 in [low, high): 52 random mantissa bits → [1,2), minus 1, scale.
double pxo_rng_gen_range_f64(pxo_rng* r, double low, double high) {
  double scale = high - low;
  for (;;) {
    uint64_t bits = (pxo_rng_next_u64(r) >> 12) | 0x3FF0000000000000ull;
    double v12;
    std::memcpy(&v12, &bits, 8);
    double v01 = v12 - 1.0;
    double res = v01 * scale + low;
    if (res < high) return res;
    scale = std::nextafter(scale, 0.0);
  }
}

// kmeans.rs:200-212
uint32_t pxo_kmeans_nearest(const float* point, const float* centroids, uint64_t dim,
                            uint64_t k, float* best_distance) {
  uint32_t best = 0;
  float bd = INFINITY;
  for (uint64_t c = 0; c < k; ++c) {
    float d = l2_sequential(point, centroids + c * dim, dim);
    if (d < bd) {
      bd = d;
      best = static_cast<uint32_t>(c);
    }
  }
  if (best_distance) *best_distance = bd;
  return best;
}

}  // extern "C"

namespace {

// kmeans.rs:146-194
void kmeans_plus_plus(const float* points, uint64_t n, uint64_t dim, uint64_t k, pxo_rng* rng,
                      float* centroids, int threads) {
  uint64_t first = pxo_rng_gen_range_usize(rng, n);
  std::memcpy(centroids, points + first * dim, dim * sizeof(float));
  std::vector<float> nearest(n);
  parallel_for(n, threads, [&](uint64_t b, uint64_t e) {
    for (uint64_t i = b; i < e; ++i) nearest[i] = l2_sequential(points + i * dim, centroids, dim);
  });
  for (uint64_t chosen = 1; chosen < k; ++chosen) {
    double total = 0.0;
    for (uint64_t i = 0; i < n; ++i) total += static_cast<double>(nearest[i]);
    uint64_t picked;
    if (total <= 0.0) {
      picked = pxo_rng_gen_range_usize(rng, n);
    } else {
      double target = pxo_rng_gen_range_f64(rng, 0.0, total);
      double cumulative = 0.0;
      picked = n - 1;
      for (uint64_t i = 0; i < n; ++i) {
        cumulative += static_cast<double>(nearest[i]);
        if (cumulative >= target) {
          picked = i;
          break;
        }
      }
    }
    float* c = centroids + chosen * dim;
    std::memcpy(c, points + picked * dim, dim * sizeof(float));
    parallel_for(n, threads, [&](uint64_t b, uint64_t e) {
      for (uint64_t i = b; i < e; ++i) {
        float d = l2_sequential(points + i * dim, c, dim);
        if (d < nearest[i]) nearest[i] = d;
      }
    });
  }
}

}  // namespace

extern "C" {

// kmeans.rs:59-143
uint64_t pxo_kmeans(const float* points, uint64_t n, uint64_t dim, uint64_t k,
                    uint64_t max_iterations, const float* init, uint64_t seed,
                    pxo_rng* rng_state, float* out_centroids, uint32_t* out_assign,
                    double* out_inertia, uint64_t* out_iterations, int threads) {
  if (dim == 0) n = 0;
  k = std::max<uint64_t>(std::min<uint64_t>(k, n), 1);
  if (n == 0) {
    std::memset(out_centroids, 0, k * dim * sizeof(float));
    *out_inertia = 0.0;
    *out_iterations = 0;
    return k;
  }
  float* centroids = out_centroids;
  if (init) {
    std::memcpy(centroids, init, k * dim * sizeof(float));
  } else {
    pxo_rng local;
    pxo_rng* rng = rng_state;
    if (!rng) {
      pxo_rng_seed_from_u64(&local, seed);
      rng = &local;
    }
    kmeans_plus_plus(points, n, dim, k, rng, centroids, threads);
  }
  std::vector<uint32_t> assignment(n, 0u);
  std::vector<float> best_d(n);
  std::vector<uint32_t> counts(k);
  std::vector<double> sums(k * dim);
  double inertia = 0.0;
  uint64_t iterations = 0;
  for (uint64_t it = 0; it < max_iterations; ++it) {
    iterations = it + 1;
    std::vector<uint32_t> fresh(n);
    parallel_for(n, threads, [&](uint64_t b, uint64_t e) {
      for (uint64_t i = b; i < e; ++i)
        fresh[i] = pxo_kmeans_nearest(points + i * dim, centroids, dim, k, &best_d[i]);
    });
    bool changed = false;
    inertia = 0.0;
    for (uint64_t i = 0; i < n; ++i) {
      inertia += static_cast<double>(best_d[i]);
      if (assignment[i] != fresh[i]) {
        assignment[i] = fresh[i];
        changed = true;
      }
    }
    if (!changed && it > 0) break;
    std::fill(counts.begin(), counts.end(), 0u);
    std::fill(sums.begin(), sums.end(), 0.0);
    for (uint64_t i = 0; i < n; ++i) {
      uint32_t c = assignment[i];
      counts[c] += 1;
      double* s = sums.data() + static_cast<uint64_t>(c) * dim;
      const float* p = points + i * dim;
      for (uint64_t d = 0; d < dim; ++d) s[d] += static_cast<double>(p[d]);
    }
    for (uint64_t c = 0; c < k; ++c) {
      if (counts[c] == 0) {
        // farthest_point (kmeans.rs:215-226) against the partially updated centroids
        uint64_t best = 0;
        float bd = -1.0f;
        std::vector<float> dist(n);
        parallel_for(n, threads, [&](uint64_t b, uint64_t e) {
          for (uint64_t i = b; i < e; ++i)
            pxo_kmeans_nearest(points + i * dim, centroids, dim, k, &dist[i]);
        });
        for (uint64_t i = 0; i < n; ++i)
          if (dist[i] > bd) {
            bd = dist[i];
            best = i;
          }
        std::memcpy(centroids + c * dim, points + best * dim, dim * sizeof(float));
        continue;
      }
      double inverse = 1.0 / static_cast<double>(counts[c]);
      for (uint64_t d = 0; d < dim; ++d)
        centroids[c * dim + d] = static_cast<float>(sums[c * dim + d] * inverse);
    }
  }
  if (out_assign) std::memcpy(out_assign, assignment.data(), n * sizeof(uint32_t));
  *out_inertia = inertia;
  *out_iterations = iterations;
  return k;
}

// product.rs:227-238
void pxo_pq_layout(uint64_t dim, uint64_t m, uint32_t* widths, uint32_t* offsets) {
  uint64_t base = dim / m, rem = dim % m, cursor = 0;
  for (uint64_t s = 0; s < m; ++s) {
    widths[s] = static_cast<uint32_t>(base + (s < rem ? 1 : 0));
    offsets[s] = static_cast<uint32_t>(cursor);
    cursor += widths[s];
  }
  offsets[m] = static_cast<uint32_t>(cursor);
}

// product.rs:198-296. Codebooks are laid out subspace-major: subspace s at
// float offset 256*offsets[s], entry c at +c*width[s].
int pxo_pq_train(const float* training, uint64_t n, uint64_t dim, uint64_t m,
                 uint64_t max_iterations, uint64_t seed, float* out_codebooks,
                 double* out_inertia, uint64_t* out_iterations, int threads) {
  if (m == 0 || m > dim || max_iterations == 0 || n == 0) return -1;
  std::vector<uint32_t> widths(m), offsets(m + 1);
  pxo_pq_layout(dim, m, widths.data(), offsets.data());
  pxo_rng rng;
  pxo_rng_seed_from_u64(&rng, seed);
  double inertia = 0.0;
  uint64_t iters = 0;
  std::vector<float> projected;
  for (uint64_t s = 0; s < m; ++s) {
    uint64_t w = widths[s], start = offsets[s];
    projected.resize(n * w);
    for (uint64_t i = 0; i < n; ++i)
      std::memcpy(projected.data() + i * w, training + i * dim + start, w * sizeof(float));
    std::vector<float> cents(256 * w);
    double ci;
    uint64_t cit;
    uint64_t produced = pxo_kmeans(projected.data(), n, w, 256, max_iterations, nullptr, 0, &rng,
                                   cents.data(), nullptr, &ci, &cit, threads);
    inertia += ci;
    iters += cit;
    float* book = out_codebooks + 256 * start;
    std::memcpy(book, cents.data(), produced * w * sizeof(float));
    for (uint64_t c = produced; c < 256; ++c)
      std::memcpy(book + c * w, cents.data() + (produced - 1) * w, w * sizeof(float));
  }
  *out_inertia = inertia;
  *out_iterations = iters;
  return 0;
}

// product.rs:361-380 + nearest_centroid :529-547
void pxo_pq_encode(const float* codebooks, uint64_t dim, uint64_t m, const float* vectors,
                   uint64_t n, uint8_t* out_codes) {
  std::vector<uint32_t> widths(m), offsets(m + 1);
  pxo_pq_layout(dim, m, widths.data(), offsets.data());
  for (uint64_t i = 0; i < n; ++i)
    for (uint64_t s = 0; s < m; ++s) {
      uint64_t w = widths[s];
      const float* x = vectors + i * dim + offsets[s];
      const float* book = codebooks + 256 * static_cast<uint64_t>(offsets[s]);
      out_codes[i * m + s] = static_cast<uint8_t>(pxo_kmeans_nearest(x, book, w, 256, nullptr));
    }
}

// product.rs decode
void pxo_pq_decode(const float* codebooks, uint64_t dim, uint64_t m, const uint8_t* codes,
                   uint64_t n, float* out) {
  std::vector<uint32_t> widths(m), offsets(m + 1);
  pxo_pq_layout(dim, m, widths.data(), offsets.data());
  for (uint64_t i = 0; i < n; ++i)
    for (uint64_t s = 0; s < m; ++s) {
      uint64_t w = widths[s];
      const float* c = codebooks + 256 * static_cast<uint64_t>(offsets[s]) + codes[i * m + s] * w;
      std::memcpy(out + i * dim + offsets[s], c, w * sizeof(float));
    }
}

// product.rs:407-439 — both tables, sequential over the subspace width.
void pxo_pq_distance_table(const float* codebooks, uint64_t dim, uint64_t m, const float* query,
                           float* out_squared, float* out_dot) {
  std::vector<uint32_t> widths(m), offsets(m + 1);
  pxo_pq_layout(dim, m, widths.data(), offsets.data());
  for (uint64_t s = 0; s < m; ++s) {
    uint64_t w = widths[s];
    const float* q = query + offsets[s];
    const float* book = codebooks + 256 * static_cast<uint64_t>(offsets[s]);
    for (uint64_t c = 0; c < 256; ++c) {
      float l2 = 0.0f, ip = 0.0f;
      for (uint64_t j = 0; j < w; ++j) {
        float d = q[j] - book[c * w + j];
        l2 += d * d;
        ip += q[j] * book[c * w + j];
      }
      if (out_squared) out_squared[s * 256 + c] = l2;
      if (out_dot) out_dot[s * 256 + c] = ip;
    }
  }
}

// product.rs:580-601
float pxo_pq_adc_squared(const float* table, uint64_t m, const uint8_t* code) {
  float sum = 0.0f;
  for (uint64_t s = 0; s < m; ++s) sum += table[s * 256 + code[s]];
  return sum;
}
float pxo_pq_adc_inner(const float* table, uint64_t m, const uint8_t* code) {
  float sum = 0.0f;
  for (uint64_t s = 0; s < m; ++s) sum += table[s * 256 + code[s]];
  return -sum;
}

// scalar.rs:141-195. Returns -1 or the first non-finite component index.
int64_t pxo_sq_train(const float* training, uint64_t n, uint64_t dim, int mode, float* out_min,
                     float* out_scale, float* out_inv_scale) {
  uint64_t groups = mode == PXO_RANGE_GLOBAL ? 1 : dim;
  std::vector<float> mn(groups, INFINITY), mx(groups, -INFINITY);
  for (uint64_t i = 0; i < n; ++i)
    for (uint64_t c = 0; c < dim; ++c) {
      float v = training[i * dim + c];
      if (!std::isfinite(v)) return static_cast<int64_t>(c);
      uint64_t g = groups == 1 ? 0 : c;
      // f32::min / f32::max on finite operands
      mn[g] = v < mn[g] ? v : mn[g];
      mx[g] = v > mx[g] ? v : mx[g];
    }
  for (uint64_t g = 0; g < groups; ++g) {
    float scale = (mx[g] - mn[g]) / 255.0f;
    out_min[g] = mn[g];
    out_scale[g] = scale;
    out_inv_scale[g] = scale > 0.0f ? 1.0f / scale : 0.0f;
  }
  return -1;
}

// scalar.rs:246-268 — level = round_half_away((v-min)*inv).clamp(0,255)
void pxo_sq_encode(const float* min, const float* inv_scale, uint64_t dim, int mode,
                   int code_type, const float* vectors, uint64_t n, uint8_t* out_codes) {
  for (uint64_t i = 0; i < n; ++i)
    for (uint64_t c = 0; c < dim; ++c) {
      uint64_t g = mode == PXO_RANGE_GLOBAL ? 0 : c;
      float x = std::round((vectors[i * dim + c] - min[g]) * inv_scale[g]);
      // clamp(0, 255) then `as u8`, which saturates and maps NaN to 0
      x = !(x >= 0.0f) ? 0.0f : (x > 255.0f ? 255.0f : x);
      uint8_t level = static_cast<uint8_t>(x);
      out_codes[i * dim + c] = code_type == PXO_CODE_I8 ? static_cast<uint8_t>(level - 128) : level;
    }
}

static inline float sq_reconstruct(const float* min, const float* scale, int mode, int code_type,
                                   uint64_t c, uint8_t byte) {
  uint64_t g = mode == PXO_RANGE_GLOBAL ? 0 : c;
  uint8_t level = code_type == PXO_CODE_I8 ? static_cast<uint8_t>(byte + 128) : byte;
  return min[g] + static_cast<float>(level) * scale[g];
}

void pxo_sq_decode(const float* min, const float* scale, uint64_t dim, int mode, int code_type,
                   const uint8_t* codes, uint64_t n, float* out) {
  for (uint64_t i = 0; i < n; ++i)
    for (uint64_t c = 0; c < dim; ++c)
      out[i * dim + c] = sq_reconstruct(min, scale, mode, code_type, c, codes[i * dim + c]);
}

// scalar.rs:298-319
float pxo_sq_asymmetric_squared_l2(const float* min, const float* scale, uint64_t dim, int mode,
                                   int code_type, const float* query, const uint8_t* code) {
  float sum = 0.0f;
  for (uint64_t c = 0; c < dim; ++c) {
    float d = query[c] - sq_reconstruct(min, scale, mode, code_type, c, code[c]);
    sum += d * d;
  }
  return sum;
}
float pxo_sq_asymmetric_inner_product(const float* min, const float* scale, uint64_t dim,
                                      int mode, int code_type, const float* query,
                                      const uint8_t* code) {
  float sum = 0.0f;
  for (uint64_t c = 0; c < dim; ++c)
    sum += query[c] * sq_reconstruct(min, scale, mode, code_type, c, code[c]);
  return -sum;
}

// ---------------------------------------------------------------------------
// Scalar-quantized filtered search (the SQ composition: the reference has no
// SQ index; its SQ path is train -> encode -> asymmetric scoring,
// crates/proxima-quantize/tests/recall.rs:139-148). Steps, per query:
//  1. the query in code space: w_c = q_c * scale_g, quantized to s8 with one
//     step per query, amax / 127: q8_c = clamp(round(w_c * (127 / amax)), -127, 127)
//     (all zero when amax == 0);
//  2. integer score S = sum_c q8_c * code_c over the I8 codes (level - 128) of
//     every accepted row. S ranks rows as the asymmetric inner product
//     (scalar.rs:298-319) does, up to the query's quantization: the per-query
//     terms sum_c q_c min_c and 128 * sum_c w_c do not depend on the row;
//  3. the `overfetch` rows of largest S, ties to the lower rank;
//  4. their exact distances (cosine 1 - dot_unrolled, inner product
//     -dot_unrolled: distance.rs:317-331, 400-402, 291-293) and the k
//     smallest by (total_cmp, id), as TopK orders them (topk.rs:63-67).
// Rows are given in rank order (ascending VectorId).
// ---------------------------------------------------------------------------
void pxo_sq_query_s8(const float* scale, uint64_t dim, int mode, const float* query, int8_t* out) {
  std::vector<float> w(dim);
  float amax = 0.0f;
  for (uint64_t c = 0; c < dim; ++c) {
    w[c] = query[c] * scale[mode == PXO_RANGE_GLOBAL ? 0 : c];
    float a = std::fabs(w[c]);
    amax = a > amax ? a : amax;
  }
  float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
  for (uint64_t c = 0; c < dim; ++c) {
    float x = std::round(w[c] * inv);
    x = x < -127.0f ? -127.0f : (x > 127.0f ? 127.0f : x);
    out[c] = static_cast<int8_t>(x);
  }
}

void pxo_sq_search(const float* scale, uint64_t dim, int mode, const int8_t* codes,
                   const float* rows, const uint64_t* ids, const uint8_t* accepted, uint64_t nrank,
                   int metric, const float* queries, uint64_t nq, uint64_t k, uint64_t overfetch,
                   uint64_t* out_ids, float* out_dist, uint32_t* out_len, int threads) {
  const uint64_t f = std::max(overfetch, k);
  parallel_for(nq, threads, [&](uint64_t qb, uint64_t qe) {
    std::vector<int8_t> q8(dim);
    std::vector<std::pair<int32_t, uint64_t>> cand;  // (-S, rank): ascending = best first
    for (uint64_t q = qb; q < qe; ++q) {
      const float* qv = queries + q * dim;
      pxo_sq_query_s8(scale, dim, mode, qv, q8.data());
      cand.clear();
      for (uint64_t r = 0; r < nrank; ++r) {
        if (accepted && !accepted[r]) continue;
        const int8_t* code = codes + r * dim;
        int32_t sum = 0;
        for (uint64_t c = 0; c < dim; ++c) sum += static_cast<int32_t>(q8[c]) * code[c];
        cand.emplace_back(-sum, r);
      }
      const uint64_t keep = std::min<uint64_t>(f, cand.size());
      std::partial_sort(cand.begin(), cand.begin() + keep, cand.end());
      TopK top(k);
      for (uint64_t i = 0; i < keep; ++i) {
        const uint64_t r = cand[i].second;
        const float dot = dot_unrolled(qv, rows + r * dim, dim);
        top.push(r, metric == PXO_COSINE ? 1.0f - dot : -dot);
      }
      auto v = top.sorted();
      for (size_t i = 0; i < v.size(); ++i) {
        out_ids[q * k + i] = ids ? ids[v[i].id] : v[i].id;
        out_dist[q * k + i] = v[i].dist;
      }
      out_len[q] = static_cast<uint32_t>(v.size());
    }
  });
}

// ivfpq.rs:1231-1243
uint32_t pxo_ivf_nearest_centroid(const float* v, const float* centroids, uint64_t dim,
                                  uint64_t count) {
  uint32_t best = 0;
  float bd = INFINITY;
  for (uint64_t l = 0; l < count; ++l) {
    float d = l2_unrolled(v, centroids + l * dim, dim);
    if (d < bd) {
      bd = d;
      best = static_cast<uint32_t>(l);
    }
  }
  return best;
}

// ivfpq.rs:828-865
void pxo_ivfpq_encode_all(const float* vectors, const uint8_t* live, uint64_t nslots,
                          uint64_t dim, const float* centroids, uint64_t nlist,
                          const float* codebooks, uint64_t m, uint32_t* out_list_of,
                          uint8_t* out_codes, int threads) {
  parallel_for(nslots, threads, [&](uint64_t b, uint64_t e) {
    std::vector<float> residual(dim);
    for (uint64_t s = b; s < e; ++s) {
      if (live && !live[s]) {
        out_list_of[s] = 0xFFFFFFFFu;
        std::memset(out_codes + s * m, 0, m);
        continue;
      }
      const float* x = vectors + s * dim;
      uint32_t l = pxo_ivf_nearest_centroid(x, centroids, dim, nlist);
      const float* c = centroids + static_cast<uint64_t>(l) * dim;
      for (uint64_t d = 0; d < dim; ++d) residual[d] = x[d] - c[d];
      pxo_pq_encode(codebooks, dim, m, residual.data(), 1, out_codes + s * m);
      out_list_of[s] = l;
    }
  });
}

// ivfpq.rs:735-825
uint64_t pxo_ivfpq_train(const float* vectors, const uint8_t* live, uint64_t nslots,
                         uint64_t dim, uint64_t nlist, uint64_t m, uint64_t max_iterations,
                         uint64_t training_sample, uint64_t seed, const float* coarse_init,
                         const float* pq_init, float* out_centroids, float* out_codebooks,
                         uint32_t* out_list_of, uint8_t* out_codes, pxo_ivf_report* report,
                         int threads) {
  std::vector<uint64_t> live_slots;
  for (uint64_t s = 0; s < nslots; ++s)
    if (!live || live[s]) live_slots.push_back(s);
  if (live_slots.empty()) return 0;
  uint64_t stride = std::max<uint64_t>((live_slots.size() + training_sample - 1) / training_sample, 1);
  std::vector<float> sample;
  for (uint64_t i = 0; i < live_slots.size(); i += stride)
    sample.insert(sample.end(), vectors + live_slots[i] * dim, vectors + (live_slots[i] + 1) * dim);
  uint64_t sampled = sample.size() / dim;
  double coarse_inertia;
  uint64_t coarse_iters;
  uint64_t produced = pxo_kmeans(sample.data(), sampled, dim, nlist, max_iterations, coarse_init,
                                 seed, nullptr, out_centroids, nullptr, &coarse_inertia,
                                 &coarse_iters, threads);
  std::vector<float> residuals(sample.size());
  for (uint64_t i = 0; i < sampled; ++i) {
    const float* x = sample.data() + i * dim;
    uint32_t l = pxo_ivf_nearest_centroid(x, out_centroids, dim, produced);
    for (uint64_t d = 0; d < dim; ++d) residuals[i * dim + d] = x[d] - out_centroids[l * dim + d];
  }
  double residual_inertia = 0.0;
  if (pq_init) {
    std::memcpy(out_codebooks, pq_init, 256 * dim * sizeof(float));
  } else {
    uint64_t pq_iters;
    pxo_pq_train(residuals.data(), sampled, dim, m, max_iterations, seed, out_codebooks,
                 &residual_inertia, &pq_iters, threads);
  }
  pxo_ivfpq_encode_all(vectors, live, nslots, dim, out_centroids, produced, out_codebooks, m,
                       out_list_of, out_codes, threads);
  if (report) {
    std::vector<uint64_t> lens(produced, 0);
    for (uint64_t s = 0; s < nslots; ++s)
      if (out_list_of[s] != 0xFFFFFFFFu) lens[out_list_of[s]]++;
    report->sampled = sampled;
    report->coarse_inertia = coarse_inertia;
    report->coarse_iterations = coarse_iters;
    report->residual_inertia = residual_inertia;
    report->populated_lists = 0;
    report->largest_list = 0;
    for (auto l : lens) {
      report->populated_lists += l > 0;
      report->largest_list = std::max(report->largest_list, l);
    }
    report->produced = produced;
  }
  return produced;
}

// ivfpq.rs:998-1110
void pxo_ivfpq_search(const float* vectors, const uint64_t* ids, const uint8_t* live,
                      uint64_t nslots, uint64_t dim, int metric, const float* centroids,
                      uint64_t nlist, const float* codebooks, uint64_t m,
                      const uint32_t* list_of, const uint8_t* codes, const float* queries,
                      uint64_t nq, uint64_t k, uint64_t nprobe, uint64_t rerank,
                      const uint64_t* bitmap, uint64_t* out_ids, float* out_dist,
                      uint32_t* out_len, int threads) {
  // lists in ascending slot order (encode_all pushes slots in order)
  std::vector<uint32_t> off(nlist + 1, 0), slot;
  for (uint64_t s = 0; s < nslots; ++s)
    if ((!live || live[s]) && list_of[s] != 0xFFFFFFFFu) ++off[list_of[s] + 1];
  for (uint64_t l = 0; l < nlist; ++l) off[l + 1] += off[l];
  slot.resize(off[nlist]);
  std::vector<uint32_t> fill(off.begin(), off.end() - 1);
  for (uint64_t s = 0; s < nslots; ++s)
    if ((!live || live[s]) && list_of[s] != 0xFFFFFFFFu) slot[fill[list_of[s]]++] = static_cast<uint32_t>(s);
  pxo_ivfpq_search_csr(vectors, ids, live, nslots, dim, metric, centroids, nlist, codebooks, m, off.data(),
                       slot.data(), codes, queries, nq, k, nprobe, rerank, bitmap, out_ids, out_dist, out_len,
                       threads);
}

// The same search over lists given as CSR (list_off[nlist+1], list_slot[]
// ascending within each list), as the index holds them between searches.
void pxo_ivfpq_search_csr(const float* vectors, const uint64_t* ids, const uint8_t* live,
                          uint64_t nslots, uint64_t dim, int metric, const float* centroids,
                          uint64_t nlist, const float* codebooks, uint64_t m,
                          const uint32_t* list_off, const uint32_t* list_slot, const uint8_t* codes,
                          const float* queries, uint64_t nq, uint64_t k, uint64_t nprobe, uint64_t rerank,
                          const uint64_t* bitmap, uint64_t* out_ids, float* out_dist,
                          uint32_t* out_len, int threads) {
  nprobe = std::min<uint64_t>(std::max<uint64_t>(nprobe, 1), std::max<uint64_t>(nlist, 1));
  std::unordered_map<uint64_t, uint64_t> by_id;
  if (ids && rerank > 0)
    for (uint64_t s = 0; s < nslots; ++s)
      if (!live || live[s]) by_id[ids[s]] = s;
  parallel_for(nq, threads, [&](uint64_t qb, uint64_t qe) {
    std::vector<float> residual(dim), table(m * 256);
    std::vector<std::pair<float, uint64_t>> coarse(nlist);
    for (uint64_t q = qb; q < qe; ++q) {
      const float* qv = queries + q * dim;
      out_len[q] = 0;
      if (k == 0) continue;
      for (uint64_t l = 0; l < nlist; ++l) coarse[l] = {l2_unrolled(qv, centroids + l * dim, dim), l};
      std::sort(coarse.begin(), coarse.end(), [](const auto& a, const auto& b) {
        int32_t ka = total_key(a.first), kb = total_key(b.first);
        return ka != kb ? ka < kb : a.second < b.second;
      });
      uint64_t shortlist = rerank > 0 ? std::max(rerank, k) : k;
      TopK top(shortlist);
      bool cosine = metric == PXO_COSINE;
      if (cosine) pxo_pq_distance_table(codebooks, dim, m, qv, nullptr, table.data());
      for (uint64_t p = 0; p < nprobe; ++p) {
        uint64_t l = coarse[p].second;
        const float* c = centroids + l * dim;
        float qdc = 0.0f;
        if (!cosine) {
          for (uint64_t d = 0; d < dim; ++d) residual[d] = qv[d] - c[d];
          pxo_pq_distance_table(codebooks, dim, m, residual.data(), table.data(), nullptr);
        } else {
          qdc = dot_unrolled(qv, c, dim);
        }
        for (uint32_t j = list_off[l]; j < list_off[l + 1]; ++j) {
          const uint32_t s = list_slot[j];
          if (!bit_set(bitmap, s)) continue;
          const uint8_t* code = codes + static_cast<uint64_t>(s) * m;
          float score = cosine ? (1.0f - qdc) + pxo_pq_adc_inner(table.data(), m, code)
                               : pxo_pq_adc_squared(table.data(), m, code);
          top.push(ids ? ids[s] : s, score);
        }
      }
      auto cand = top.sorted();
      if (rerank == 0 || vectors == nullptr) {
        uint64_t n = std::min<uint64_t>(k, cand.size());
        for (uint64_t i = 0; i < n; ++i) {
          out_ids[q * k + i] = cand[i].id;
          out_dist[q * k + i] = cand[i].dist;
        }
        out_len[q] = static_cast<uint32_t>(n);
        continue;
      }
      // rerank against the exact vectors; ids map back to slots
      TopK exact(k);
      for (const Hit& h : cand) {
        uint64_t slot = h.id;
        if (ids) {
          auto it = by_id.find(h.id);
          if (it == by_id.end()) continue;
          slot = it->second;
        }
        exact.push(h.id, space_distance(metric, qv, vectors + slot * dim, dim));
      }
      auto v = exact.sorted();
      for (size_t i = 0; i < v.size(); ++i) {
        out_ids[q * k + i] = v[i].id;
        out_dist[q * k + i] = v[i].dist;
      }
      out_len[q] = static_cast<uint32_t>(v.size());
    }
  });
}

// crc32c_append (crates/proxima-store/src/crc.rs:29-79): the byte table of
// the reflected Castagnoli polynomial, one byte per step, register !crc in
// and inverted out.
uint32_t pxo_crc32c_append(uint32_t crc, const uint8_t* bytes, uint64_t len) {
  static const std::vector<uint32_t> table = [] {
    std::vector<uint32_t> t(256);
    for (uint32_t b = 0; b < 256; ++b) {
      uint32_t r = b;
      for (int bit = 0; bit < 8; ++bit) r = (r & 1u) ? (r >> 1) ^ 0x82F63B78u : r >> 1;
      t[b] = r;
    }
    return t;
  }();
  uint32_t r = ~crc;
  for (uint64_t i = 0; i < len; ++i) r = table[(r ^ bytes[i]) & 0xFFu] ^ (r >> 8);
  return ~r;
}

}  // extern "C"
