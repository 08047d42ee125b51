/*
 * proxima_cuda.h — C ABI of libproxima_cuda.so, the B200 (sm_100a) backend for
 * Proxima's nearest-neighbour hot path.
 *
 * Plain C types only: pointers, sizes, integer codes. No C++ exception and no
 * CUDA error crosses this boundary; every entry point returns a pxc_status and,
 * when `err` is non-NULL, fills a pxc_error describing the failure.
 *
 * Each entry point names the reference interface (Liona-orph/proxima, Rust)
 * it replaces. The Rust side keeps its types and calls these through a thin
 * FFI crate (`proxima-cuda`) that declares these functions and owns the
 * handles.
 *
 * Conventions shared by all entry points:
 *  - Host pointers are borrowed for the duration of the call and copied; no
 *    pointer is retained after return.
 *  - Vectors are row-major f32, `dim` floats per row. "Prepared" means
 *    VectorSpace::prepare has been applied (validated; cosine rows normalised),
 *    crates/proxima-core/src/space.rs:130-138.
 *  - Results are ordered ascending by (f32::total_cmp(distance), id), the
 *    order of SearchResult (crates/proxima-core/src/topk.rs:63-67). Result row
 *    q occupies out[q*k .. q*k+k); out_len[q] says how many entries are valid.
 *  - Filters are bitmaps over slots: bit (s & 63) of word s/64 set means slot s
 *    is accepted; NULL accepts all (the AcceptAll filter,
 *    crates/proxima-index/src/index.rs:43-50).
 *  - Handles are used by one thread at a time for mutation (sync/destroy); the
 *    search entry points may be called concurrently on one handle.
 */
#ifndef PROXIMA_CUDA_H
#define PROXIMA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes: one per ProximaError variant (crates/proxima-core/src/error.rs:37-160),
 *      plus device and timeout failures, which map to ProximaError::Internal ---- */
typedef int32_t pxc_status;
#define PXC_OK 0
#define PXC_DIMENSION_MISMATCH 1 /* a = expected, b = actual */
#define PXC_UNKNOWN_ID 2         /* a = id */
#define PXC_DUPLICATE_ID 3       /* a = id */
#define PXC_CAPACITY 4           /* a = limit, detail = what */
#define PXC_NON_FINITE 5         /* a = component index */
#define PXC_CORRUPTION 6
#define PXC_CONFIGURATION 7      /* parameter, a = value, detail = reason */
#define PXC_INTERNAL 8
#define PXC_IO 9
#define PXC_DEVICE 10            /* a CUDA error; detail holds its text */
#define PXC_TIMEOUT 11           /* a device-side bounded wait gave up */

typedef struct pxc_error {
  int32_t code;
  uint64_t a;
  uint64_t b;
  char parameter[32];
  char detail[256];
} pxc_error;

/* metric codes, in the declaration order of proxima_core::Metric
 * (crates/proxima-core/src/distance.rs:90-135) */
#define PXC_EUCLIDEAN 0
#define PXC_COSINE 1
#define PXC_INNER_PRODUCT 2
#define PXC_MANHATTAN 3

/* Largest k a search accepts: check_k (crates/proxima-index/src/index.rs:212-224). */
#define PXC_MAX_K (1u << 24)

/* ---- version / capability ---- */
/* Returns the ABI version (major << 16 | minor). */
uint32_t pxc_abi_version(void);

/* ---- context: one CUDA device, its streams and scratch ----
 * Replaces nothing in the reference (which is single-threaded CPU code); it
 * owns the device state every handle below is created on. Exactly one device
 * per context: multi-GPU runs use one process (and one context) per GPU and
 * exchange candidates over the context's NCCL communicator
 * (pxc_ctx_init_comm, pxc_flat_search_sharded, pxc_topk_exchange). */
typedef struct pxc_ctx pxc_ctx;
pxc_status pxc_ctx_create(const int* devices, int n_devices, pxc_ctx** out, pxc_error* err);
void pxc_ctx_destroy(pxc_ctx* ctx);
/* Device-side wait limit in milliseconds for kernels with bounded spins
 * (default 2000). A wait that runs out returns PXC_TIMEOUT. */
pxc_status pxc_ctx_set_wait_limit(pxc_ctx* ctx, uint32_t milliseconds, pxc_error* err);

/* ---- observability ----
 * Count of kernels this library launched on the context since creation
 * (every scan, selection, merge and mirror-maintenance kernel). */
uint64_t pxc_ctx_launch_count(const pxc_ctx* ctx);
/* When on, the searches record CUDA events around their dominant scan kernel
 * on the launching stream; pxc_flat_last_scan_ms reads the last duration
 * (milliseconds, synchronising on the end event). Off by default. */
pxc_status pxc_ctx_set_profiling(pxc_ctx* ctx, int32_t on, pxc_error* err);
/* Diagnostic switches for tests, off by default; no production caller sets
 * them. "sq_candidate_cap" (>= 0) shrinks the SQ threshold pass's candidate
 * buffers so that its exact fallback runs; "sq_spec_rank" (>= 1) forces the SQ
 * speculative admission rank; "kmeans_exact" (0/1) assigns k-means points
 * without the tensor-core screen; "kmeans_trace" (0/1) prints per-iteration
 * counters to stderr; "flat_group_sample" (n >= 1) fixes the share 1/n of
 * the rows that the flat search at 32 < k <= 128 samples for its admission
 * bound (default, or negative: 800 / k), 0 skips the sample pass; "flat_collect_cap"
 * (default 2048, rounded up to a power of two in [32, 2048]) sets the
 * per-query candidate slots of that search's single collect launch, 0 runs
 * the group launches instead. A negative SQ cap or rank restores the default.
 * Unknown names are PXC_CONFIGURATION. */
pxc_status pxc_ctx_set_option(pxc_ctx* ctx, const char* name, int64_t value, pxc_error* err);

/* ---- FlatIndex: exact filtered top-k ----
 * Replaces the scan loop of FlatIndex::search
 * (crates/proxima-index/src/flat.rs:153-169) and adds the batched form
 * search_batch. The device holds a mirror of the VectorStore
 * (crates/proxima-core/src/storage.rs:100-115): slot-major prepared rows,
 * the VectorId of each slot and a live flag. */
typedef struct pxc_flat pxc_flat;
pxc_status pxc_flat_create(pxc_ctx* ctx, uint32_t dim, int32_t metric, pxc_flat** out,
                           pxc_error* err);
void pxc_flat_destroy(pxc_flat* h);
/* Copy slots [slot_begin, slot_begin + nslots) of the host store into the
 * mirror: `rows` nslots*dim prepared floats, `ids` the VectorId per slot
 * (NULL means id == slot), `live` one byte per slot (NULL means all live).
 * Slots beyond the current high-water mark grow the mirror. Rows must be
 * finite (PXC_NON_FINITE otherwise, a = flat component index). */
pxc_status pxc_flat_sync(pxc_flat* h, const float* rows, const uint64_t* ids,
                         const uint8_t* live, uint64_t slot_begin, uint64_t nslots,
                         pxc_error* err);
/* Shrink the mirror to `nslots` slots (after VectorStore::clear or compaction). */
pxc_status pxc_flat_truncate(pxc_flat* h, uint64_t nslots, pxc_error* err);
/* Number of live slots in the mirror. */
uint64_t pxc_flat_len(const pxc_flat* h);
/* Batched exact search with HOST buffers: `queries` nq*dim prepared floats,
 * `bitmap` over slots or NULL; outputs nq*k ids and distances and nq lengths.
 * Dimension is fixed at create; k <= PXC_MAX_K. */
pxc_status pxc_flat_search(pxc_flat* h, const float* queries, uint32_t nq, uint32_t k,
                           const uint64_t* bitmap, uint64_t* out_ids, float* out_dist,
                           uint32_t* out_len, pxc_error* err);
/* The same search with the filter given as MetadataFilter conditions
 * (see pxc_columns below) over `cols`, the handle's metadata columns indexed by
 * slot: the accepted set is computed on the device, no bitmap crosses the
 * boundary. HOST queries and outputs. */
typedef struct pxc_columns pxc_columns;
typedef struct pxc_condition pxc_condition;
typedef struct pxc_operand pxc_operand;
pxc_status pxc_flat_search_where(pxc_flat* h, pxc_columns* cols, const pxc_condition* conds, uint32_t ncond,
                                 const pxc_operand* operands, uint32_t noperands, const float* queries, uint32_t nq,
                                 uint32_t k, uint64_t* out_ids, float* out_dist, uint32_t* out_len, pxc_error* err);
/* Same, with DEVICE buffers on the context's device, ordered on `stream`
 * (a cudaStream_t; NULL = the context's stream). The call waits on the
 * stream for small host decisions (whether the queries are integers in
 * [0,255]; with 32 < k <= 128, which queries overflowed their candidate
 * slots or were not proven exact by the row-group launches)
 * and returns with the result kernels enqueued; the caller synchronises the
 * stream before reading the outputs. */
pxc_status pxc_flat_search_device(pxc_flat* h, const float* d_queries, uint32_t nq,
                                  uint32_t k, const uint64_t* d_bitmap, uint64_t* d_out_ids,
                                  float* d_out_dist, uint32_t* d_out_len, void* stream,
                                  pxc_error* err);
/* Which scan kernel the next search will use: 1 = tensor-core u8 (every live
 * row and the queries are integers in [0,255] under euclidean, so the u8
 * product is exact; k <= 128); 2 = tensor-core f16 screen of K2_KT = 32
 * candidates per query, re-ranked with the exact f32 distance and proven per
 * query (any other store under euclidean, cosine or inner product with
 * dim <= 128, for unfiltered searches with k <= 24; unproven queries run on the
 * fp32 scan); 0 = fp32 reference-order scan. Diagnostic only. */
int32_t pxc_flat_path(const pxc_flat* h);
/* Duration of the last search's scan kernel (K1 or K1g), with profiling on;
 * -1 when not recorded. */
float pxc_flat_last_scan_ms(pxc_flat* h);
/* Queries of the last search that the first tensor-core pass did not settle
 * and that were answered again: with 32 < k <= 128 on the u8 path, those
 * whose collect-launch candidates overflowed (answered by the row-group
 * launches) plus those the row-group proof could not settle (32 or more of
 * their top k in one group; answered by the fp32 scan); on the f16 screen,
 * those whose candidates' k-th exact distance was not provably ahead of every
 * row the screen left out (fp32 scan); 0 otherwise. */
uint32_t pxc_flat_last_redone(const pxc_flat* h);

/* Allocation-free variant of pxc_flat_search_device. No counterpart in the
 * reference: it exists for callers that cannot allocate device memory (a host
 * runtime that has reserved the device for its own pool, or a serving loop
 * that cannot afford the device-wide synchronisation of cudaMalloc/cudaFree).
 * Its scratch is one file-scope device array of about 8.6 MiB, held on every
 * GPU that loads the library. Limits: nq <= 2048, k <= 16, dim <= 256, a
 * euclidean store of integers in [0,255] (the tensor-core scan), queries of
 * integers in [0,255], and a device mirror already built by an earlier
 * pxc_flat_len or search (PXC_CAPACITY / PXC_CONFIGURATION otherwise). The
 * first call on a device looks up the array's address. Each call
 * synchronises `stream` twice (after checking that the queries are integers,
 * and at the end) and returns after its work has finished. Calls share the
 * array; within a process they are serialised.
 * Device buffers. */
pxc_status pxc_flat_search_noalloc(pxc_flat* h, const float* d_queries, uint32_t nq, uint32_t k,
                                   uint64_t* d_out_ids, float* d_out_dist, uint32_t* d_out_len,
                                   void* stream, pxc_error* err);

/* ---- typed metadata filters on the device ----
 * MetadataFilter (crates/proxima-server/src/filter.rs:58-75, 216-256)
 * compiled to conditions over typed device columns and evaluated by one
 * thread per slot into the bitmap over slots that every search entry point
 * takes (pxc_flat_search_device, pxc_ivfpq_search_device, pxc_sq_search_device
 * and the sharded forms): the per-slot host closure pass is gone. A column
 * holds one MetadataValue per slot as a type tag and a 64-bit payload: Int
 * the i64, Float the f64 bits, Bool 0/1, Text a code the caller assigns per
 * distinct string (equal strings, equal codes). Tags follow MetadataValue's
 * declaration order (crates/proxima-core/src/metadata.rs:21-31). */
#define PXC_VALUE_ABSENT 0
#define PXC_VALUE_TEXT 1
#define PXC_VALUE_INT 2
#define PXC_VALUE_FLOAT 3
#define PXC_VALUE_BOOL 4
/* Condition operators, in the order of filter.rs's Condition enum. */
#define PXC_COND_EQ 0
#define PXC_COND_NE 1
#define PXC_COND_GT 2
#define PXC_COND_GE 3
#define PXC_COND_LT 4
#define PXC_COND_LE 5
#define PXC_COND_IN 6
#define PXC_COND_EXISTS 7
/* One condition on one column. eq / ne: (tag, value) is the operand; gt, gte,
 * lt, lte: a numeric bound (tag INT or FLOAT); in: `count` operands starting at
 * operands[value]; exists: value != 0 means exists:true. All conditions must
 * hold; an absent field fails all but exists:false. */
struct pxc_condition {
  uint32_t column;
  uint32_t op;
  uint32_t tag;
  uint32_t count;
  int64_t value;
};
struct pxc_operand {
  uint32_t tag;
  uint32_t reserved;
  int64_t value;
};
pxc_status pxc_columns_create(pxc_ctx* ctx, pxc_columns** out, pxc_error* err);
void pxc_columns_destroy(pxc_columns* cols);
/* Slots [slot_begin, slot_begin + nslots) of column `column` (< 4096): HOST
 * tags and payloads. Slots never written read as absent. */
pxc_status pxc_columns_set(pxc_columns* cols, uint32_t column, const uint8_t* tags, const int64_t* values,
                           uint64_t slot_begin, uint64_t nslots, pxc_error* err);
/* Forget every slot at or beyond nslots (after the store shrank). */
pxc_status pxc_columns_truncate(pxc_columns* cols, uint64_t nslots, pxc_error* err);
/* The accepted slots among [0, nslots) as a DEVICE bitmap of ceil(nslots/64)
 * words (bit s & 63 of word s/64), ordered on `stream`; conditions and operands
 * are HOST arrays. Returns after the bitmap is written. */
pxc_status pxc_columns_eval(pxc_columns* cols, uint64_t nslots, const pxc_condition* conds, uint32_t ncond,
                            const pxc_operand* operands, uint32_t noperands, uint64_t* d_bitmap, void* stream,
                            pxc_error* err);

/* ---- multi-GPU: the context's communicator and the candidate exchange ----
 * The reference is single-process; this is the data-parallel form of its
 * search: every rank holds a shard of the rows (with their global
 * VectorIds), searches all queries on it, and one NCCL allgather over NVLink
 * carries the k candidates per query to every rank, where they are merged by
 * (total_cmp(distance), id) (TopK::push over the union,
 * crates/proxima-core/src/topk.rs:119-138). NCCL is loaded at run time
 * (libnccl.so.2); without it these entry points return PXC_CONFIGURATION. */
#define PXC_COMM_ID_BYTES 128
/* A fresh communicator id (ncclGetUniqueId). Rank 0 creates it and hands the
 * 128 bytes to every rank by the job's own means (MPI, a TCP store, ...). */
pxc_status pxc_comm_unique_id(uint8_t out[PXC_COMM_ID_BYTES], pxc_error* err);
/* Joins the context to the job's communicator (ncclCommInitRank; collective
 * over the ranks). nranks == 1 needs no id traffic and makes the exchanges
 * below local merges. timeout_ms bounds every later wait on the exchange: on
 * expiry, or an asynchronous NCCL error, the communicator is aborted and the
 * call returns PXC_TIMEOUT / PXC_DEVICE. Every rank must issue the exchanges
 * in the same order. */
pxc_status pxc_ctx_init_comm(pxc_ctx* ctx, const uint8_t id[PXC_COMM_ID_BYTES], int32_t nranks, int32_t rank,
                             uint32_t timeout_ms, pxc_error* err);
int32_t pxc_ctx_comm_size(const pxc_ctx* ctx);
int32_t pxc_ctx_comm_rank(const pxc_ctx* ctx);
/* FlatIndex::search over a row-sharded store: this rank's handle holds its
 * shard (global VectorIds as ids); every rank passes the same prepared
 * queries. Local exact search, one packed allgather (ids, distances, lengths
 * of k candidates per query in a single buffer), merge: every rank receives
 * the global top-k, equal to one unsharded search. DEVICE buffers; returns
 * after the exchange has finished. nranks * k <= 8192. */
pxc_status pxc_flat_search_sharded(pxc_flat* h, const float* d_queries, uint32_t nq, uint32_t k,
                                   const uint64_t* d_bitmap, uint64_t* d_out_ids, float* d_out_dist,
                                   uint32_t* d_out_len, void* stream, pxc_error* err);
/* The same exchange for any local top-k_in lists (nq x k_in ids and
 * distances, nq lengths; DEVICE buffers), each sorted by (total_cmp, id) as
 * every search here returns them, e.g. an SQ or IVF-PQ shard's answer:
 * allgather over the communicator and merge into the global top-k. */
pxc_status pxc_topk_exchange(pxc_ctx* ctx, const uint64_t* d_ids, const float* d_dist, const uint32_t* d_lens,
                             uint32_t nq, uint32_t k_in, uint32_t k, uint64_t* d_out_ids, float* d_out_dist,
                             uint32_t* d_out_len, void* stream, pxc_error* err);

/* ---- multi-GPU merge ----
 * After each rank searched its own row shard, an allgather leaves `nparts`
 * candidate lists per query on every rank: part p of query q at
 * [(p*nq + q)*k_in, ...), lengths at lens[p*nq + q]. Merges them into the
 * top-k by (total_cmp(distance), id). DEVICE buffers. This is TopK::push over
 * the union (crates/proxima-core/src/topk.rs:119-138). */
pxc_status pxc_topk_merge(pxc_ctx* ctx, const uint64_t* d_ids, const float* d_dist,
                          const uint32_t* d_lens, uint32_t nparts, uint32_t nq, uint32_t k_in,
                          uint32_t k, uint64_t* d_out_ids, float* d_out_dist,
                          uint32_t* d_out_len, void* stream, pxc_error* err);

/* ---- ChaCha8Rng ----
 * The generator the reference's training draws from: rand_chacha 0.3.1's
 * ChaCha8Rng (crates/proxima-quantize/src/kmeans.rs:150,167,169,
 * product.rs:247, crates/proxima-index/src/ivfpq.rs:770), carried across the
 * boundary as the three values rand_chacha exposes: get_seed() (32 bytes),
 * get_stream() and get_word_pos() (a u128 count of u32 words, below 2^68).
 * A Rust caller passes its generator with
 *   pxc_rng { seed: rng.get_seed(), stream: rng.get_stream(),
 *             word_pos_lo: pos as u64, word_pos_hi: (pos >> 64) as u64 }
 * and afterwards restores it with set_stream + set_word_pos. These run on the
 * host (no device work). */
typedef struct pxc_rng {
  uint8_t seed[32];
  uint64_t stream;
  uint64_t word_pos_lo;
  uint64_t word_pos_hi;
} pxc_rng;
/* ChaCha8Rng::seed_from_u64(state) (rand_core 0.6.4: PCG32 expansion of the
 * u64 into the 32-byte seed), stream 0, word position 0. */
pxc_status pxc_rng_seed_from_u64(uint64_t state, pxc_rng* out, pxc_error* err);
/* n successive RngCore::next_u32 draws; advances `rng`. */
pxc_status pxc_rng_next_u32(pxc_rng* rng, uint32_t* out, uint64_t n, pxc_error* err);
/* Rng::gen_range(0..bound) for usize (rand 0.8); bound >= 1. Advances `rng`. */
pxc_status pxc_rng_gen_index(pxc_rng* rng, uint64_t bound, uint64_t* out, pxc_error* err);
/* Rng::gen_range(low..high) for f64 (rand 0.8); low < high, finite span. */
pxc_status pxc_rng_gen_f64(pxc_rng* rng, double low, double high, double* out, pxc_error* err);
/* The ChaCha block function with `rounds` rounds (8 is ChaCha8Rng's; 20 is
 * RFC 8439's): 16 words for (key, 64-bit block counter, 64-bit stream).
 * Exposed so the generator can be checked against published known answers. */
pxc_status pxc_chacha_block(const uint32_t key[8], uint64_t counter, uint64_t stream, uint32_t rounds,
                            uint32_t out[16], pxc_error* err);

/* ---- k-means ----
 * Replaces proxima_quantize::kmeans (crates/proxima-quantize/src/kmeans.rs:59-143),
 * which ProductQuantizer::train (product.rs:247-274) and IvfPqIndex::train
 * (crates/proxima-index/src/ivfpq.rs:771-777) call. Same algorithm, same
 * results: k is clamped to max(min(k, n), 1); Lloyd iterations with argmin
 * ties to the lower centroid index, f64 sums in point order, empty clusters
 * re-seeded at the farthest point, early stop when no assignment changes
 * (the stopping pass is counted). */
typedef struct pxc_kmeans_info {
  uint32_t k;          /* centroids produced (the clamp above) */
  uint32_t iterations; /* Clustering::iterations */
  double inertia;      /* Clustering::inertia (the last assignment pass) */
  uint32_t path;       /* 0: exact CUDA-core assignment; 1: tensor-core screening + exact re-scoring */
  uint32_t reseeded;   /* empty clusters re-seeded */
  uint64_t rescanned;  /* point assignments settled by a full exact scan */
  uint32_t screen_passes; /* tensor-core screening launches (CAND passes) */
  float screen_ms;     /* their summed device time, when profiling is on (pxc_ctx_set_profiling) */
} pxc_kmeans_info;

/* points: n x dim f32 row-major (HOST). init: NULL for the reference's
 * k-means++ seeding (kmeans.rs:146-194) drawn from `rng`, the caller's
 * ChaCha8Rng state, which is advanced in place exactly as the reference's
 * `&mut ChaCha8Rng` is (kmeans.rs:59-65); or k_eff x dim initial centroids
 * (an added option: the reference always seeds with k-means++), in which case
 * `rng` is neither read nor advanced and may be NULL. out_centroids: room for
 * k_eff x dim; out_assign (nullable): n cluster indices. info (nullable).
 * dim <= 512; points must be finite (PXC_NON_FINITE, a = flat element index).
 * n == 0 returns k_eff zero centroids without drawing. */
pxc_status pxc_kmeans(pxc_ctx* ctx, const float* points, uint64_t n, uint32_t dim, uint32_t k,
                      uint32_t max_iterations, const float* init, pxc_rng* rng,
                      float* out_centroids, uint32_t* out_assign, pxc_kmeans_info* info,
                      pxc_error* err);
/* The same with DEVICE buffers on `stream` (NULL: the context stream). */
pxc_status pxc_kmeans_device(pxc_ctx* ctx, const float* d_points, uint64_t n, uint32_t dim,
                             uint32_t k, uint32_t max_iterations, const float* d_init,
                             pxc_rng* rng, float* d_out_centroids, uint32_t* d_out_assign,
                             pxc_kmeans_info* info, void* stream, pxc_error* err);

/* ---- ProductQuantizer ----
 * crates/proxima-quantize/src/product.rs. Codebooks are 256 x dim floats in
 * ProductQuantizer::codebooks' layout: subspace-major, subspace s holding 256
 * codewords of width[s] floats at 256 * offset[s], widths dim / m with the
 * remainder spread over the leading subspaces (product.rs:227-238).
 * 1 <= m <= dim <= 1024 (PXC_CONFIGURATION "subspaces" otherwise). */
/* ProductQuantizer::train (product.rs:198-296) on n x dim HOST training rows:
 * one ChaCha8Rng::seed_from_u64(seed) stream advanced across subspaces,
 * kmeans(projection, width, 256, max_iterations, rng) per subspace (on the
 * device, as pxc_kmeans), codebooks padded to 256 entries by repeating the
 * last centroid. out_inertia / out_iterations (nullable) are
 * training_inertia / training_iterations. n == 0 is PXC_CONFIGURATION
 * ("training"); a non-finite component is PXC_NON_FINITE (a = its index
 * within the vector). */
pxc_status pxc_pq_train(pxc_ctx* ctx, const float* training, uint64_t n, uint32_t dim, uint32_t m,
                        uint32_t max_iterations, uint64_t seed, float* out_codebooks, double* out_inertia,
                        uint64_t* out_iterations, pxc_error* err);
/* Same with DEVICE training rows and codebook output, on `stream`. */
pxc_status pxc_pq_train_device(pxc_ctx* ctx, const float* d_training, uint64_t n, uint32_t dim, uint32_t m,
                               uint32_t max_iterations, uint64_t seed, float* d_out_codebooks, double* out_inertia,
                               uint64_t* out_iterations, void* stream, pxc_error* err);
/* ProductQuantizer::encode_into (product.rs:361-380) for n vectors: per
 * subspace the codeword with the smallest sequential squared distance, ties
 * to the lower index (nearest_centroid, :529-547). HOST buffers; out_codes
 * n x m bytes. */
pxc_status pxc_pq_encode(pxc_ctx* ctx, const float* codebooks, uint32_t dim, uint32_t m, const float* vectors,
                         uint64_t n, uint8_t* out_codes, pxc_error* err);
/* Same with DEVICE codebooks, vectors and codes, on `stream`. */
pxc_status pxc_pq_encode_device(pxc_ctx* ctx, const float* d_codebooks, uint32_t dim, uint32_t m,
                                const float* d_vectors, uint64_t n, uint8_t* d_out_codes, void* stream,
                                pxc_error* err);
/* ProductQuantizer::decode (product.rs:387-398): the chosen codewords
 * concatenated, n x dim floats. HOST buffers. */
pxc_status pxc_pq_decode(pxc_ctx* ctx, const float* codebooks, uint32_t dim, uint32_t m, const uint8_t* codes,
                         uint64_t n, float* out, pxc_error* err);
/* ProductQuantizer::distance_table (product.rs:407-439) for nq queries:
 * out_squared / out_dot are nq x m x 256 floats, entry (q, s, c) at
 * (q * m + s) * 256 + c, each the sequential sum over the subspace width of
 * (q - c)^2 or q * c. DistanceTable::squared_l2 / inner_product
 * (product.rs:580-601) are then m lookups per code. HOST buffers. */
pxc_status pxc_pq_tables(pxc_ctx* ctx, const float* codebooks, uint32_t dim, uint32_t m, const float* queries,
                         uint32_t nq, float* out_squared, float* out_dot, pxc_error* err);
/* Same with DEVICE buffers, on `stream`. */
pxc_status pxc_pq_tables_device(pxc_ctx* ctx, const float* d_codebooks, uint32_t dim, uint32_t m,
                                const float* d_queries, uint32_t nq, float* d_out_squared, float* d_out_dot,
                                void* stream, pxc_error* err);

/* kmeans over points sharded across the ranks of the context's communicator
 * (pxc_ctx_init_comm): this rank's n points (DEVICE, n x dim) are its
 * consecutive range of the global point order, rank by rank. Every rank
 * passes the same k x dim DEVICE init (the injected-init mode of pxc_kmeans;
 * the sharded form has no k-means++ seeding) and receives the same
 * centroids; out_assign (nullable) gets its own points' clusters. Each
 * iteration exchanges, over the communicator, the inertia and changed flag
 * of the assignment pass and the per-cluster f64 sums and counts (folded in
 * rank order), and for every empty cluster the ranks' farthest points (the
 * global one wins, ties to the lower global index), so the iteration count,
 * assignments and re-seeding follow kmeans.rs:59-143 over the whole set;
 * centroids equal the unsharded run's whenever the per-cluster sums are exact
 * and otherwise agree within rounding. Every rank needs n >= 1. */
pxc_status pxc_kmeans_sharded(pxc_ctx* ctx, const float* d_points, uint64_t n, uint32_t dim, uint32_t k,
                              uint32_t max_iterations, const float* d_init, float* d_out_centroids,
                              uint32_t* d_out_assign, pxc_kmeans_info* info, void* stream, pxc_error* err);

/* ---- IvfPqIndex ----
 * The device side of IvfPqIndex (crates/proxima-index/src/ivfpq.rs): coarse
 * centroids + product-quantizer codebooks, inverted lists of PQ codes in
 * ascending slot order, and the full-precision store for reranking.
 * Euclidean and cosine (the metrics whose scoring search_prepared defines). */
typedef struct pxc_ivfpq pxc_ivfpq;
/* nlist coarse centroids, m subspaces of 256 centroids (widths as
 * ProductQuantizer::train lays them out, product.rs:227-238). dim <= 1024, m <= 64. */
pxc_status pxc_ivfpq_create(pxc_ctx* ctx, uint32_t dim, int32_t metric, uint32_t nlist, uint32_t m,
                            pxc_ivfpq** out, pxc_error* err);
void pxc_ivfpq_destroy(pxc_ivfpq* h);
/* IvfPqIndex::from_parts (ivfpq.rs:624-717): centroids nlist*dim, codebooks
 * 256*dim (ProductQuantizer::codebooks layout, subspace-major). HOST buffers. */
pxc_status pxc_ivfpq_set_parts(pxc_ivfpq* h, const float* centroids, const float* codebooks,
                               pxc_error* err);
/* The slot store: `vectors` nslots*dim prepared floats (NULL: no reranking,
 * the retain_vectors=false case), `ids` the VectorId per slot (NULL: id ==
 * slot), `live` one byte per slot (NULL: all live). HOST buffers. Clears the lists. */
pxc_status pxc_ivfpq_set_store(pxc_ivfpq* h, const float* vectors, const uint64_t* ids,
                               const uint8_t* live, uint64_t nslots, pxc_error* err);
/* Same, with the vectors in DEVICE memory (copied); ids and live on the host. */
pxc_status pxc_ivfpq_set_store_device(pxc_ivfpq* h, const float* d_vectors, const uint64_t* ids,
                                      const uint8_t* live, uint64_t nslots, pxc_error* err);
/* Duration of the last search's scan kernel (K5/K6) when it ran as one batch
 * with profiling on; -1 otherwise. */
float pxc_ivfpq_last_scan_ms(pxc_ivfpq* h);
/* PQ codes the last search scored, summed over its queries (synchronising). */
uint64_t pxc_ivfpq_last_scanned(pxc_ivfpq* h);
/* The lists from per-slot assignments (list_of, 0xFFFFFFFF = unassigned)
 * and codes (nslots*m bytes): IvfPqIndex's list_of / codes. HOST buffers. */
pxc_status pxc_ivfpq_set_codes(pxc_ivfpq* h, const uint32_t* list_of, const uint8_t* codes,
                               pxc_error* err);
/* encode_all (ivfpq.rs:828-865): every live slot's list (nearest centroid by
 * squared_euclidean, ties to the lower index) and PQ code of its residual,
 * lists in ascending slot order. Needs parts and the vectors. */
pxc_status pxc_ivfpq_encode_all(pxc_ivfpq* h, pxc_error* err);
/* IvfPqIndex::train (ivfpq.rs:735-825): the stride sample of the live slots
 * (every ceil(live/training_sample)-th), coarse k-means (k-means++ from
 * ChaCha8Rng::seed_from_u64(seed)), PQ codebooks on the sample's residuals
 * with a fresh stream of the same seed advanced across subspaces
 * (product.rs:198-296), then encode_all. The list count becomes what k-means
 * produced (nlist clamped to the sample size). */
typedef struct pxc_ivfpq_report {
  uint64_t sampled;          /* TrainingReport::sampled */
  double coarse_inertia;     /* TrainingReport::coarse_inertia */
  uint64_t coarse_iterations;
  double residual_inertia;   /* ProductQuantizer::training_inertia */
  uint64_t populated_lists;
  uint64_t largest_list;
  uint64_t produced;         /* lists (centroids) produced */
  uint64_t pq_iterations;    /* ProductQuantizer::training_iterations */
} pxc_ivfpq_report;
pxc_status pxc_ivfpq_train(pxc_ivfpq* h, uint64_t training_sample, uint32_t max_iterations, uint64_t seed,
                           pxc_ivfpq_report* report, pxc_error* err);
/* IvfPqIndex::parts (ivfpq.rs:606-617): copies out (each nullable) centroids
 * nlist*dim, codebooks 256*dim, list_of nslots, codes nslots*m, and nlist. */
pxc_status pxc_ivfpq_get_parts(pxc_ivfpq* h, float* centroids, float* codebooks, uint32_t* list_of,
                               uint8_t* codes, uint32_t* out_nlist, pxc_error* err);
/* IvfPqIndex::search_with_nprobe (ivfpq.rs:981-1110) for a batch of prepared
 * queries: nprobe clamped to [1, nlist] (<= 128), shortlist max(rerank, k)
 * (<= 4096), bitmap over slots or NULL. HOST buffers. */
pxc_status pxc_ivfpq_search(pxc_ivfpq* h, const float* queries, uint32_t nq, uint32_t k,
                            uint32_t nprobe, uint32_t rerank, const uint64_t* bitmap,
                            uint64_t* out_ids, float* out_dist, uint32_t* out_len, pxc_error* err);
/* The same search with the filter given as MetadataFilter conditions over
 * the handle's metadata columns (pxc_columns), evaluated on the device. HOST
 * queries and outputs. */
pxc_status pxc_ivfpq_search_where(pxc_ivfpq* h, pxc_columns* cols, const pxc_condition* conds, uint32_t ncond,
                                  const pxc_operand* operands, uint32_t noperands, const float* queries, uint32_t nq,
                                  uint32_t k, uint32_t nprobe, uint32_t rerank, uint64_t* out_ids, float* out_dist,
                                  uint32_t* out_len, pxc_error* err);
/* Same with DEVICE buffers on `stream` (NULL: the context stream); returns
 * once enqueued. */
pxc_status pxc_ivfpq_search_device(pxc_ivfpq* h, const float* d_queries, uint32_t nq, uint32_t k,
                                   uint32_t nprobe, uint32_t rerank, const uint64_t* d_bitmap,
                                   uint64_t* d_out_ids, float* d_out_dist, uint32_t* d_out_len,
                                   void* stream, pxc_error* err);

/* The owner-computes form of pxc_flat_search_sharded, for batches whose
 * queries each belong to one rank: every rank searches all nq DEVICE queries
 * on its shard, then each rank receives from every rank only the candidates of
 * its own query slice [nq*rank/nranks, nq*(rank+1)/nranks) (grouped NCCL sends
 * and receives, k candidates per query) and merges them; the outputs hold that
 * slice's results (pxc_ctx_owned_range gives its bounds). Every rank calls it
 * with the same nq and queries; returns after the exchange has finished. */
pxc_status pxc_flat_search_sharded_owned(pxc_flat* h, const float* d_queries, uint32_t nq, uint32_t k,
                                         const uint64_t* d_bitmap, uint64_t* d_out_ids, float* d_out_dist,
                                         uint32_t* d_out_len, void* stream, pxc_error* err);
/* The slice [*begin, *begin + *count) of nq queries this context's rank owns. */
void pxc_ctx_owned_range(const pxc_ctx* ctx, uint32_t nq, uint32_t* begin, uint32_t* count);

/* search_with_nprobe over an index whose rows are sharded across the ranks of
 * the context's communicator: every rank holds the same parts (centroids,
 * codebooks) and the lists of its own rows (global VectorIds as ids), probes
 * the same nprobe lists on its shard, re-ranks its own shortlist of
 * max(rerank, k), and one packed allgather + merge gives every rank the
 * global top-k: the union of the ranks' answers ordered by (total_cmp, id).
 * DEVICE buffers; returns after the exchange has finished. */
pxc_status pxc_ivfpq_search_sharded(pxc_ivfpq* h, const float* d_queries, uint32_t nq, uint32_t k, uint32_t nprobe,
                                    uint32_t rerank, const uint64_t* d_bitmap, uint64_t* d_out_ids, float* d_out_dist,
                                    uint32_t* d_out_len, void* stream, pxc_error* err);

/* ---- Snapshots ----
 * The snapshot file of crates/proxima-store/src/snapshot.rs (format version 1,
 * little-endian codec of crates/proxima-store/src/codec.rs):
 *   "PROXSNAP" | u32 version | u32 0x01020304 | u32 0 | u64 body_len | body | u32 crc32c(body)
 * An IVF-PQ body (kind 3, snapshot.rs:150-186) holds the space, the
 * IvfPqConfig, the slot ids, the metadata, then vectors, codes, list_of,
 * centroids and codebooks as u32-counted arrays, and the TrainingReport.
 * Errors: PXC_CORRUPTION with `parameter` naming the structure (as
 * ProximaError::Corruption), PXC_CONFIGURATION for a body whose values
 * IvfPqIndex::new rejects or that exceeds this build's device limits. */

/* crc32c_append (crates/proxima-store/src/crc.rs:64-79): CRC-32C
 * (Castagnoli) continued over `len` more HOST bytes; (0, b, n) is crc32c(b). */
uint32_t pxc_crc32c_append(uint32_t crc, const void* bytes, uint64_t len);
/* crc32c(A || B) from crc32c(A), crc32c(B) and the length of B. */
uint32_t pxc_crc32c_combine(uint32_t crc_a, uint32_t crc_b, uint64_t len_b);
/* crc32c of `len` DEVICE bytes, computed on the device, returned in *out
 * (synchronises `stream`; NULL: the context stream). `d_bytes` may have any
 * alignment but must lie in an allocation that starts 16-byte aligned
 * (cudaMalloc and the caching allocators): the kernel reads from it rounded
 * down to 16 bytes. */
pxc_status pxc_crc32c_device(pxc_ctx* ctx, const void* d_bytes, uint64_t len, uint32_t* out, void* stream,
                             pxc_error* err);

/* IvfPqConfig (crates/proxima-index/src/ivfpq.rs:104-150) as the snapshot
 * records it (snapshot.rs:469-479). */
typedef struct pxc_ivfpq_config {
  uint32_t nlist;
  uint32_t subspaces;
  uint32_t nprobe;
  uint32_t rerank;
  uint64_t seed;
  uint32_t max_iterations;
  uint32_t training_sample;
  uint64_t train_threshold;
  uint32_t retain_vectors; /* 0 or 1 */
  uint32_t reserved;
} pxc_ivfpq_config;

/* What a snapshot says about itself (snapshot.rs:96-110 SnapshotHeader, and
 * for IVF-PQ the rest of the body's small fields). */
typedef struct pxc_snapshot_info {
  uint32_t format_version;
  uint32_t kind;             /* 1 flat, 2 hnsw, 3 ivfpq */
  uint32_t dim;
  int32_t metric;            /* PXC_EUCLIDEAN .. PXC_MANHATTAN */
  uint64_t body_bytes;
  uint64_t nslots;           /* entries of the id table */
  uint64_t live;             /* slots holding an id: the index's len() */
  uint64_t metadata_offset;  /* IVF-PQ: byte offset in the image of the metadata section (its u32 count first) */
  uint64_t metadata_bytes;
  pxc_ivfpq_config config;   /* IVF-PQ only */
  uint32_t trained;          /* the centroids and codebooks are present */
  uint32_t lists;            /* centroids / dim when trained, else config.nlist */
  uint32_t has_vectors;      /* the full-precision vectors are present */
  uint32_t has_report;
  pxc_ivfpq_report report;   /* TrainingReport when has_report (produced and pq_iterations 0) */
} pxc_snapshot_info;

/* peek (snapshot.rs:271-299) of a HOST image: header, checksum (on the host),
 * space and kind. An IVF-PQ body is decoded and checked in full, as decode
 * does; of a flat or HNSW body only the id table is read. */
pxc_status pxc_snapshot_peek(const uint8_t* bytes, uint64_t len, pxc_snapshot_info* info, pxc_error* err);
/* decode (snapshot.rs:192-269) of an IVF-PQ snapshot straight into a new
 * device index: the HOST image's arrays go by one copy each into the
 * handle's device buffers, the checksum joins the host pieces' CRC with the
 * arrays' CRC computed on the device, and the id ranks and the inverted
 * lists are built on the device (IvfPqIndex::from_parts, ivfpq.rs:624-717).
 * The errors and their precedence are decode's. Metadata stays in the image:
 * info->metadata_offset / metadata_bytes locate it. *out is NULL on error. */
pxc_status pxc_ivfpq_snapshot_load(pxc_ctx* ctx, const uint8_t* bytes, uint64_t len, pxc_ivfpq** out,
                                   pxc_snapshot_info* info, pxc_error* err);
/* encode (snapshot.rs:120-200) of a device index into the HOST buffer `out`
 * of `capacity` bytes; *out_len = the snapshot's size (out NULL: size only).
 * `config` is recorded as given (subspaces must equal the index's); `report`
 * NULL records none. `metadata` is the encoded metadata section (u32 count =
 * the slot count, then per slot the codec's Metadata with keys sorted;
 * codec.rs:170-200), NULL for empty metadata on every slot. Slots without a
 * live id are written as (0, 0). The arrays' CRC is computed on the device. */
pxc_status pxc_ivfpq_snapshot_save(pxc_ivfpq* h, const pxc_ivfpq_config* config, const pxc_ivfpq_report* report,
                                   const uint8_t* metadata, uint64_t metadata_bytes, uint8_t* out, uint64_t capacity,
                                   uint64_t* out_len, pxc_error* err);

/* ---- ScalarQuantizer ----
 * crates/proxima-quantize/src/scalar.rs. Range modes and code types in the
 * declaration order of RangeMode / CodeType. */
#define PXC_RANGE_GLOBAL 0
#define PXC_RANGE_PER_DIMENSION 1
#define PXC_CODE_U8 0
#define PXC_CODE_I8 1
/* ScalarQuantizer::train (scalar.rs:141-195) on n x dim HOST training rows:
 * per group (1 under Global, dim under PerDimension) the observed min, scale
 * = (max - min) / 255 and inverse_scale = scale > 0 ? 1 / scale : 0.
 * Bit-identical to the reference's sequential fold, including the sign of a
 * zero bound. n == 0 is PXC_CONFIGURATION ("training"); a non-finite value is
 * PXC_NON_FINITE with a = its index within the vector. */
pxc_status pxc_sq_train(pxc_ctx* ctx, const float* training, uint64_t n, uint32_t dim, int32_t mode,
                        float* out_min, float* out_scale, float* out_inv_scale, pxc_error* err);
/* Same with DEVICE training rows (outputs on the host), on `stream`. */
pxc_status pxc_sq_train_device(pxc_ctx* ctx, const float* d_training, uint64_t n, uint32_t dim,
                               int32_t mode, float* out_min, float* out_scale, float* out_inv_scale,
                               void* stream, pxc_error* err);
/* The observed (min, max) per group of DEVICE training rows, before the
 * scale is formed: what a trainer sharded over ranks combines. Folding the
 * ranks' values in rank order with `v < min` / `v > max` reproduces the
 * single-pass result exactly. Outputs on the host. */
pxc_status pxc_sq_ranges_device(pxc_ctx* ctx, const float* d_training, uint64_t n, uint32_t dim,
                                int32_t mode, float* out_min, float* out_max, void* stream,
                                pxc_error* err);
/* ScalarQuantizer::encode_into (scalar.rs:246-268) for n vectors: HOST
 * buffers, out_codes n x dim bytes (U8 levels or I8 level - 128). */
pxc_status pxc_sq_encode(pxc_ctx* ctx, const float* min, const float* inv_scale, uint32_t dim,
                         int32_t mode, int32_t code_type, const float* vectors, uint64_t n,
                         uint8_t* out_codes, pxc_error* err);
/* Same with DEVICE vectors and codes (the range table on the host). */
pxc_status pxc_sq_encode_device(pxc_ctx* ctx, const float* min, const float* inv_scale, uint32_t dim,
                                int32_t mode, int32_t code_type, const float* d_vectors, uint64_t n,
                                uint8_t* d_out_codes, void* stream, pxc_error* err);
/* ScalarQuantizer::decode (scalar.rs:270-296): min + level * scale. HOST buffers. */
pxc_status pxc_sq_decode(pxc_ctx* ctx, const float* min, const float* scale, uint32_t dim, int32_t mode,
                         int32_t code_type, const uint8_t* codes, uint64_t n, float* out,
                         pxc_error* err);

/* ScalarQuantizer::asymmetric_squared_l2 (metric PXC_EUCLIDEAN) or
 * asymmetric_inner_product (PXC_INNER_PRODUCT, and PXC_COSINE on prepared
 * vectors) (scalar.rs:298-327) for every pair of nq HOST queries and n HOST
 * codes: out[q * n + i], the reference's sequential sum over components with
 * reconstruct = min + level * scale, bit for bit. nq <= 524280. */
pxc_status pxc_sq_asymmetric(pxc_ctx* ctx, const float* min, const float* scale, uint32_t dim, int32_t mode,
                             int32_t code_type, int32_t metric, const float* queries, uint32_t nq,
                             const uint8_t* codes, uint64_t n, float* out, pxc_error* err);
/* Same with DEVICE queries, codes and output (the range table on the host),
 * on `stream`. */
pxc_status pxc_sq_asymmetric_device(pxc_ctx* ctx, const float* min, const float* scale, uint32_t dim, int32_t mode,
                                    int32_t code_type, int32_t metric, const float* d_queries, uint32_t nq,
                                    const uint8_t* d_codes, uint64_t n, float* d_out, void* stream, pxc_error* err);

/* ---- SQ filtered search ----
 * No counterpart index in the reference: its SQ path is train -> encode ->
 * asymmetric scoring (crates/proxima-quantize/tests/recall.rs:139-148,
 * scalar.rs:298-319). The device index holds the prepared rows (the re-rank
 * store), their I8 codes, the VectorIds and integer metadata columns, and
 * answers "top-k by the metric among the rows the filter accepts" as an int8
 * over-fetch followed by an exact re-rank: the query in code space is
 * quantized to s8 (one step per query, max |q_c * scale_c| / 127), the
 * `overfetch` rows with the largest s8 . code score (ties to the lower id)
 * are re-scored with VectorSpace::distance (cosine 1 - dot_unrolled, inner
 * product -dot_unrolled) and the k smallest by (total_cmp, id) returned.
 * Cosine and inner product; dim <= 1024. */
typedef struct pxc_sq pxc_sq;
/* A metadata condition lo <= value <= hi on an integer column (set with
 * pxc_sq_set_column); a slot without the field fails it. The typed form of
 * an Int filter (crates/proxima-server/src/filter.rs:58-75); e.g.
 * year >= 2027 is {column, 0, 2027, INT64_MAX}. */
typedef struct pxc_int_range {
  uint32_t column;
  uint32_t reserved;
  int64_t lo;
  int64_t hi;
} pxc_int_range;
pxc_status pxc_sq_create(pxc_ctx* ctx, uint32_t dim, int32_t metric, pxc_sq** out, pxc_error* err);
void pxc_sq_destroy(pxc_sq* h);
/* ScalarQuantizer::from_parts-style: a trained range table (groups entries
 * each). Re-encodes the store when one is set. HOST buffers. */
pxc_status pxc_sq_set_quantizer(pxc_sq* h, int32_t mode, const float* min, const float* scale,
                                const float* inv_scale, pxc_error* err);
pxc_status pxc_sq_get_quantizer(pxc_sq* h, int32_t* mode, float* min, float* scale, float* inv_scale,
                                pxc_error* err);
/* ScalarQuantizer::train over the live stored rows (slot order), then encode. */
pxc_status pxc_sq_train_store(pxc_sq* h, int32_t mode, pxc_error* err);
/* The slot store: nslots*dim prepared floats, VectorId per slot (NULL: id ==
 * slot), live byte per slot (NULL: all live). Clears the metadata columns and
 * re-encodes when a quantizer is set. HOST buffers. */
pxc_status pxc_sq_set_store(pxc_sq* h, const float* vectors, const uint64_t* ids, const uint8_t* live,
                            uint64_t nslots, pxc_error* err);
/* Same with the vectors in DEVICE memory (copied); ids and live on the host. */
pxc_status pxc_sq_set_store_device(pxc_sq* h, const float* d_vectors, const uint64_t* ids,
                                   const uint8_t* live, uint64_t nslots, pxc_error* err);
/* Integer metadata column `column`: one value per slot, `present` one byte
 * per slot (NULL: every slot has the field). HOST buffers. */
pxc_status pxc_sq_set_column(pxc_sq* h, uint32_t column, const int64_t* values, const uint8_t* present,
                             pxc_error* err);
/* Live rows in the store. */
uint64_t pxc_sq_len(const pxc_sq* h);
/* The stored I8 codes per slot (nslots x dim; dead slots zero). HOST buffer. */
pxc_status pxc_sq_get_codes(pxc_sq* h, uint8_t* out_codes, pxc_error* err);
/* Batched filtered search with HOST buffers: `queries` nq*dim prepared
 * floats, `bitmap` over slots or NULL, `ranges` nranges (<= 8) conditions
 * ANDed with it; max(overfetch, k) <= 2048. Outputs nq*k ids/distances and
 * nq lengths. */
pxc_status pxc_sq_search(pxc_sq* h, const float* queries, uint32_t nq, uint32_t k, uint32_t overfetch,
                         const uint64_t* bitmap, const pxc_int_range* ranges, uint32_t nranges,
                         uint64_t* out_ids, float* out_dist, uint32_t* out_len, pxc_error* err);
/* Same with DEVICE queries, bitmap and outputs (`ranges` stays a host array),
 * ordered on `stream` (NULL: the context stream). Returns after the work has
 * finished: the accepted-row count sizes the scan. */
pxc_status pxc_sq_search_device(pxc_sq* h, const float* d_queries, uint32_t nq, uint32_t k,
                                uint32_t overfetch, const uint64_t* d_bitmap, const pxc_int_range* ranges,
                                uint32_t nranges, uint64_t* d_out_ids, float* d_out_dist,
                                uint32_t* d_out_len, void* stream, pxc_error* err);
/* Device time of the last search's scan (K12 passes and selection) when it
 * ran as one batch with profiling on; -1 otherwise. */
float pxc_sq_last_scan_ms(pxc_sq* h);
/* Rows the last search's filter accepted. */
uint64_t pxc_sq_last_accepted(const pxc_sq* h);
/* Queries of the last search whose speculative admission key admitted too
 * few rows and that were scanned again with the safe key. */
uint32_t pxc_sq_last_retried(const pxc_sq* h);
/* Queries of the last search whose candidates overflowed the over-fetch
 * buffer and were answered by the exact chunked fallback. */
uint32_t pxc_sq_last_fallback(const pxc_sq* h);

#ifdef __cplusplus
}
#endif
#endif /* PROXIMA_CUDA_H */
