/*
 * pxo.h — CPU oracle for the Proxima nearest-neighbour hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is
 * compared against; it is never the thing measured or shipped. Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
 * may load it.
 *
 * It restates, in C++17 built with -ffp-contract=off and no fast-math, the
 * arithmetic of the Rust reference (Liona-orph/proxima) for:
 *   crates/proxima-core/src/{distance.rs,space.rs,topk.rs}
 *   crates/proxima-index/src/{flat.rs,ivfpq.rs,recall.rs,index.rs}
 *   crates/proxima-quantize/src/{kmeans.rs,product.rs,scalar.rs}
 * Every function names the reference file:line it follows.
 *
 * Parity status: the deterministic arithmetic (distance kernels, TopK order,
 * flat search, Lloyd iterations from a given init, PQ encode/tables/ADC, SQ,
 * IVF-PQ search from given parts) is pinned against the reference's own
 * known-answer tests (tests/test_oracle_*.py). The k-means++ seeding depends on
 * rand_chacha 0.3.1 / rand_core 0.6.4 / rand 0.8.x, whose source is absent;
 * it is restated from the published ChaCha and PCG32 algorithms and its draws
 * are "parity unpinned" (no golden draw exists in the reference tests).
 */
#ifndef PXO_H
#define PXO_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* metric codes, same order as proxima_core::Metric (distance.rs:90) */
enum { PXO_EUCLIDEAN = 0, PXO_COSINE = 1, PXO_INNER_PRODUCT = 2, PXO_MANHATTAN = 3 };

/* ---- distance.rs ---- */
float pxo_squared_euclidean(const float* a, const float* b, uint64_t dim);
float pxo_squared_euclidean_scalar(const float* a, const float* b, uint64_t dim);
float pxo_dot(const float* a, const float* b, uint64_t dim);
float pxo_manhattan(const float* a, const float* b, uint64_t dim);
float pxo_cosine(const float* a, const float* b, uint64_t dim);
float pxo_cosine_normalized(const float* a, const float* b, uint64_t dim);
float pxo_normalize_in_place(float* v, uint64_t dim);
/* VectorSpace::distance on prepared operands (space.rs:148-156) */
float pxo_space_distance(int metric, const float* a, const float* b, uint64_t dim);
/* VectorSpace::prepare on n rows (space.rs:130-138); returns -1 on success or
 * the index of the first non-finite component (row-major flat index). */
int64_t pxo_prepare(int metric, float* rows, uint64_t n, uint64_t dim);

/* ---- flat.rs: exact filtered top-k over a slot-major store ----
 * data: nslots*dim prepared rows; ids: nslots VectorIds; live: nslots flags;
 * bitmap: optional accept bitmap over slots (bit s of word s/64).
 * Results per query are written at [q*k, q*k+len), len to out_len[q]. */
void pxo_flat_search(const float* data, const uint64_t* ids, const uint8_t* live,
                     uint64_t nslots, uint64_t dim, int metric,
                     const float* queries, uint64_t nq, uint64_t k,
                     const uint64_t* bitmap, uint64_t* out_ids, float* out_dist,
                     uint32_t* out_len, int threads);

/* ---- recall.rs ---- */
float pxo_recall_overlap(const uint64_t* exact, uint32_t exact_len,
                         const uint64_t* approx, uint32_t approx_len);

/* ---- rand restatement (ChaCha8 + PCG32 seed expansion + rand 0.8 ranges) ---- */
typedef struct pxo_rng { uint32_t key[8]; uint64_t counter; uint32_t buf[64]; uint32_t index; } pxo_rng;
/* the ChaCha block function: key, 64-bit counter (words 12-13), 64-bit stream (14-15), rounds */
void pxo_chacha_block(const uint32_t key[8], uint64_t counter, uint64_t stream, int rounds, uint32_t out[16]);
void pxo_rng_seed_from_u64(pxo_rng* r, uint64_t seed);
uint32_t pxo_rng_next_u32(pxo_rng* r);
uint64_t pxo_rng_next_u64(pxo_rng* r);
uint64_t pxo_rng_gen_range_usize(pxo_rng* r, uint64_t n);
double pxo_rng_gen_range_f64(pxo_rng* r, double low, double high);

/* ---- kmeans.rs ----
 * init: NULL → k-means++ from ChaCha8(seed) (unpinned), else k*dim centroids.
 * rng_state: optional pxo_rng advanced in place (used by PQ training to share
 * one stream across subspaces). Returns k actually used. */
uint64_t pxo_kmeans(const float* points, uint64_t n, uint64_t dim, uint64_t k,
                    uint64_t max_iterations, const float* init, uint64_t seed,
                    pxo_rng* rng_state, float* out_centroids, uint32_t* out_assign,
                    double* out_inertia, uint64_t* out_iterations, int threads);
/* nearest() with sequential sums (kmeans.rs:200-212) */
uint32_t pxo_kmeans_nearest(const float* point, const float* centroids, uint64_t dim,
                            uint64_t k, float* best_distance);

/* ---- product.rs ---- */
void pxo_pq_layout(uint64_t dim, uint64_t m, uint32_t* widths, uint32_t* offsets);
int pxo_pq_train(const float* training, uint64_t n, uint64_t dim, uint64_t m,
                 uint64_t max_iterations, uint64_t seed, float* out_codebooks,
                 double* out_inertia, uint64_t* out_iterations, int threads);
void pxo_pq_encode(const float* codebooks, uint64_t dim, uint64_t m,
                   const float* vectors, uint64_t n, uint8_t* out_codes);
void pxo_pq_decode(const float* codebooks, uint64_t dim, uint64_t m,
                   const uint8_t* codes, uint64_t n, float* out);
void pxo_pq_distance_table(const float* codebooks, uint64_t dim, uint64_t m,
                           const float* query, float* out_squared, float* out_dot);
float pxo_pq_adc_squared(const float* table_squared, uint64_t m, const uint8_t* code);
float pxo_pq_adc_inner(const float* table_dot, uint64_t m, const uint8_t* code);

/* ---- scalar.rs ---- */
enum { PXO_RANGE_GLOBAL = 0, PXO_RANGE_PER_DIMENSION = 1 };
enum { PXO_CODE_U8 = 0, PXO_CODE_I8 = 1 };
int64_t pxo_sq_train(const float* training, uint64_t n, uint64_t dim, int mode,
                     float* out_min, float* out_scale, float* out_inv_scale);
void pxo_sq_encode(const float* min, const float* inv_scale, uint64_t dim, int mode,
                   int code_type, const float* vectors, uint64_t n, uint8_t* out_codes);
void pxo_sq_decode(const float* min, const float* scale, uint64_t dim, int mode,
                   int code_type, const uint8_t* codes, uint64_t n, float* out);
float pxo_sq_asymmetric_squared_l2(const float* min, const float* scale, uint64_t dim,
                                   int mode, int code_type, const float* query,
                                   const uint8_t* code);
float pxo_sq_asymmetric_inner_product(const float* min, const float* scale, uint64_t dim,
                                      int mode, int code_type, const float* query,
                                      const uint8_t* code);

/* SQ composition (no reference index): query quantization to s8 and the
 * over-fetch + exact re-rank search over I8 codes in rank order. */
void pxo_sq_query_s8(const float* scale, uint64_t dim, int mode, const float* query, int8_t* out);
void pxo_sq_search(const float* scale, uint64_t dim, int mode, const int8_t* codes,
                   const float* rows, const uint64_t* ids, const uint8_t* accepted, uint64_t nrank,
                   int metric, const float* queries, uint64_t nq, uint64_t k, uint64_t overfetch,
                   uint64_t* out_ids, float* out_dist, uint32_t* out_len, int threads);

/* ---- ivfpq.rs ---- */
/* nearest_centroid with 8-lane L2 (ivfpq.rs:1231-1243) */
uint32_t pxo_ivf_nearest_centroid(const float* v, const float* centroids, uint64_t dim,
                                  uint64_t count);
/* IvfPqIndex::train over live slots (ivfpq.rs:735-825) + encode_all (:828-865).
 * centroid_init: optional nlist*dim coarse init (skips k-means++ for the coarse
 * stage; PQ codebooks still use their own seeded stream unless pq_init given).
 * Outputs: centroids (nlist*dim), codebooks (256*dim), list_of (nslots),
 * codes (nslots*m). Returns produced list count. */
typedef struct pxo_ivf_report {
  uint64_t sampled, coarse_iterations, populated_lists, largest_list, produced;
  double coarse_inertia, residual_inertia;
} pxo_ivf_report;
uint64_t pxo_ivfpq_train(const float* vectors, const uint8_t* live, uint64_t nslots,
                         uint64_t dim, uint64_t nlist, uint64_t m, uint64_t max_iterations,
                         uint64_t training_sample, uint64_t seed,
                         const float* coarse_init, const float* pq_init,
                         float* out_centroids, float* out_codebooks, uint32_t* out_list_of,
                         uint8_t* out_codes, pxo_ivf_report* report, int threads);
/* encode_all given trained parts */
void pxo_ivfpq_encode_all(const float* vectors, const uint8_t* live, uint64_t nslots,
                          uint64_t dim, const float* centroids, uint64_t nlist,
                          const float* codebooks, uint64_t m, uint32_t* out_list_of,
                          uint8_t* out_codes, int threads);
/* search_prepared (ivfpq.rs:998-1110) for nq prepared queries. Lists are the
 * slots with list_of[s]==l in ascending slot order. vectors may be NULL when
 * rerank==0. metric is PXO_EUCLIDEAN or PXO_COSINE. */
void pxo_ivfpq_search_csr(const float* vectors, const uint64_t* ids, const uint8_t* live,
                          uint64_t nslots, uint64_t dim, int metric, const float* centroids,
                          uint64_t nlist, const float* codebooks, uint64_t m,
                          const uint32_t* list_off, const uint32_t* list_slot, const uint8_t* codes,
                          const float* queries, uint64_t nq, uint64_t k, uint64_t nprobe, uint64_t rerank,
                          const uint64_t* bitmap, uint64_t* out_ids, float* out_dist,
                          uint32_t* out_len, int threads);
void pxo_ivfpq_search(const float* vectors, const uint64_t* ids, const uint8_t* live,
                      uint64_t nslots, uint64_t dim, int metric, const float* centroids,
                      uint64_t nlist, const float* codebooks, uint64_t m,
                      const uint32_t* list_of, const uint8_t* codes, const float* queries,
                      uint64_t nq, uint64_t k, uint64_t nprobe, uint64_t rerank,
                      const uint64_t* bitmap, uint64_t* out_ids, float* out_dist,
                      uint32_t* out_len, int threads);

/* crc32c_append (crates/proxima-store/src/crc.rs:64-79), byte at a time. */
uint32_t pxo_crc32c_append(uint32_t crc, const uint8_t* bytes, uint64_t len);

#ifdef __cplusplus
}
#endif
#endif
