// snapshot.cu — IVF-PQ snapshots loaded and saved straight between a host
// byte image of the file and the device, and CRC-32C computed on the device.
//
// File format (crates/proxima-store/src/snapshot.rs:1-15, 120-283, the codec
// of crates/proxima-store/src/codec.rs, all little-endian):
//
//   "PROXSNAP" | u32 version (1) | u32 0x01020304 | u32 0 | u64 body_len
//   | body | u32 crc32c(body)
//   body (IVF-PQ, kind 3) = u32 dim, u8 metric tag | u8 kind | config
//     (u32 nlist, u32 subspaces, u32 nprobe, u32 rerank, u64 seed,
//      u32 max_iterations, u32 training_sample, u64 train_threshold,
//      u8 retain_vectors)
//     | u32 n, n x (u8 present, u64 id) | u32 n, n x metadata
//     | f32[] vectors | u8[] codes | u32[] list_of | f32[] centroids
//     | f32[] codebooks | u8 has_report [u32 sampled, f64 coarse_inertia,
//       u32 coarse_iterations, f64 residual_inertia, u32 populated_lists,
//       u32 largest_list]
//   where T[] is a u32 element count then the elements.
//
// Load: the host walks the small sections (space, config, ids, metadata,
// the length prefixes), each large array goes by one copy from the image
// into its device buffer, and the body's checksum is the combination of the
// host pieces' CRC and the device arrays' CRC computed on the GPU: the host
// never reads the arrays. The list CSR and the id ranks are built on the
// device (stable radix sorts). Save is the mirror: the host writes the small
// sections, the arrays come back by one copy each, and their CRC is taken on
// the device before the copy.
//
// Error precedence follows the reference's decode (snapshot.rs:192-269,
// 331-380): header checks, then the checksum, then the body's own errors in
// reading order, then IvfPqIndex::from_parts (ivfpq.rs:624-717), then
// trailing bytes. A body error found before the checksum is known is
// reported only after a host CRC of the whole body has matched.
#include <cub/cub.cuh>

#include <algorithm>
#include <cmath>
#include <memory>
#include <vector>

#include "common.cuh"
#include "hostcopy.cuh"
#include "ivfpq.cuh"

namespace pxc {
namespace crc {

// ---------------------------------------------------------------------------
// CRC-32C (crc.rs:29-78): Castagnoli polynomial, bit-reflected, register
// initialised to !crc and inverted on output. The register update is linear
// over GF(2), so with f(r, D) the register after D from r:
//   f(r, A||B) = S_|B|(f(r, A)) ^ f(0, B)     (S_n: n zero bytes)
//   crc32c(D) = ~(S_|D|(~0) ^ f(0, D))
//   crc32c(A||B) = S_|B|(crc32c(A)) ^ crc32c(B)
// and f(0, 0^k || D) = f(0, D): leading zero bytes do not move a zero
// register. The device kernel splits D into runs that threads fold
// independently and joins them with S; the S operators are 32x32 bit
// matrices (column i = the image of bit i), applied either as four 256-entry
// byte tables or, for one vector per warp, as a XOR reduction over lanes.
// ---------------------------------------------------------------------------
constexpr uint32_t POLY = 0x82F63B78u;
constexpr int UNIT = 512;     // bytes one thread folds per step: two 256-byte halves, two chains
constexpr int THREADS = 512;  // threads of the step kernel (16 warps)
constexpr uint64_t STEP = (uint64_t)UNIT * THREADS;
constexpr int LEVELS = 10;    // operators S_{UNIT << l}, l = 0..9 (the last one is S_STEP)
constexpr int OPS = LEVELS + 1;  // and S_{UNIT / 2}, which joins the halves (stored first)
constexpr int SLICE_WORDS = 4 * 256;
constexpr int OP_WORDS = 4 * 256;
constexpr int DEV_WORDS = SLICE_WORDS + OPS * OP_WORDS;
// slicing tables with one copy per shared-memory bank, then the operators
constexpr size_t STEP_SMEM = (size_t)SLICE_WORDS * 32 * 4 + (size_t)OPS * OP_WORDS * 4;
static_assert(THREADS == 512, "the step kernel's tree is 5 lane levels and 4 warp levels");
static_assert((UNIT << (LEVELS - 1)) == (int)STEP, "the last operator joins whole steps");

struct Mat {
  uint32_t c[32];
};

inline uint32_t apply(const Mat& m, uint32_t v) {
  uint32_t r = 0;
  for (int i = 0; v; ++i, v >>= 1)
    if (v & 1u) r ^= m.c[i];
  return r;
}
inline Mat compose(const Mat& a, const Mat& b) {  // a after b
  Mat r;
  for (int i = 0; i < 32; ++i) r.c[i] = apply(a, b.c[i]);
  return r;
}

struct Tables {
  uint32_t t[8][256];  // slicing-by-8; t[0] is crc.rs's byte table
  Mat pow2[64];        // S_{2^k}
  std::vector<uint32_t> dev;
  Tables() {
    for (uint32_t b = 0; b < 256; ++b) {
      uint32_t r = b;
      for (int k = 0; k < 8; ++k) r = (r >> 1) ^ (POLY & (0u - (r & 1u)));
      t[0][b] = r;
    }
    for (int k = 1; k < 8; ++k)
      for (int b = 0; b < 256; ++b) t[k][b] = (t[k - 1][b] >> 8) ^ t[0][t[k - 1][b] & 0xFFu];
    for (int i = 0; i < 32; ++i) {
      const uint32_t v = 1u << i;
      pow2[0].c[i] = (v >> 8) ^ t[0][v & 0xFFu];
    }
    for (int k = 1; k < 64; ++k) pow2[k] = compose(pow2[k - 1], pow2[k - 1]);
    dev.assign(DEV_WORDS, 0);
    for (int k = 0; k < 4; ++k)
      for (int b = 0; b < 256; ++b) dev[k * 256 + b] = t[k][b];
    op_table(matrix(UNIT / 2), dev.data() + SLICE_WORDS);
    for (int l = 0; l < LEVELS; ++l)
      op_table(matrix((uint64_t)UNIT << l), dev.data() + SLICE_WORDS + (l + 1) * OP_WORDS);
  }
  Mat matrix(uint64_t n) const {  // S_n
    Mat r;
    for (int i = 0; i < 32; ++i) r.c[i] = 1u << i;
    for (int k = 0; n; ++k, n >>= 1)
      if (n & 1u) r = compose(pow2[k], r);
    return r;
  }
  uint32_t shift(uint32_t v, uint64_t n) const {
    for (int k = 0; n; ++k, n >>= 1)
      if (n & 1u) v = apply(pow2[k], v);
    return v;
  }
  static void op_table(const Mat& m, uint32_t* out) {
    for (int k = 0; k < 4; ++k)
      for (uint32_t b = 0; b < 256; ++b) out[k * 256 + b] = apply(m, b << (8 * k));
  }
};

const Tables& tables() {
  static const Tables t;
  return t;
}

// The register after `n` bytes from `r` (no inversion), slicing-by-8.
uint32_t update(uint32_t r, const uint8_t* p, uint64_t n) {
  const auto& T = tables().t;
  while (n && (reinterpret_cast<uintptr_t>(p) & 7u)) {
    r = (r >> 8) ^ T[0][(r ^ *p++) & 0xFFu];
    --n;
  }
  while (n >= 8) {
    uint32_t lo, hi;
    std::memcpy(&lo, p, 4);
    std::memcpy(&hi, p + 4, 4);
    lo ^= r;
    r = T[7][lo & 0xFFu] ^ T[6][(lo >> 8) & 0xFFu] ^ T[5][(lo >> 16) & 0xFFu] ^ T[4][lo >> 24] ^ T[3][hi & 0xFFu] ^
        T[2][(hi >> 8) & 0xFFu] ^ T[1][(hi >> 16) & 0xFFu] ^ T[0][hi >> 24];
    p += 8;
    n -= 8;
  }
  while (n--) r = (r >> 8) ^ T[0][(r ^ *p++) & 0xFFu];
  return r;
}
uint32_t append(uint32_t crc, const void* p, uint64_t n) { return ~update(~crc, static_cast<const uint8_t*>(p), n); }
uint32_t combine(uint32_t a, uint32_t b, uint64_t len_b) { return tables().shift(a, len_b) ^ b; }

// ---- device ----
__device__ __forceinline__ uint32_t op_apply(const uint32_t* op, uint32_t v) {
  return op[v & 0xFFu] ^ op[256 + ((v >> 8) & 0xFFu)] ^ op[512 + ((v >> 16) & 0xFFu)] ^ op[768 + (v >> 24)];
}
// One slicing-by-4 step from the bank-private copy of the tables (entry
// (k, e) of this lane at rep[(k * 256 + e) * 32]).
__device__ __forceinline__ uint32_t slice4(const uint32_t* rep, uint32_t x) {
  return rep[(768 + (x & 0xFFu)) * 32] ^ rep[(512 + ((x >> 8) & 0xFFu)) * 32] ^
         rep[(256 + ((x >> 16) & 0xFFu)) * 32] ^ rep[(x >> 24) * 32];
}
__device__ __forceinline__ uint32_t keep_from(uint32_t w, int first) {  // zero bytes [0, first) of w
  return first <= 0 ? w : first >= 4 ? 0u : (w & ~((1u << (8 * first)) - 1u));
}

// Step kernel: every thread folds one UNIT-byte run per step, f(0, run), as
// two independent chains over its halves (64 bytes of each per iteration,
// the next iteration's bytes loaded before the current ones are folded),
// joined by S_{UNIT/2}; a lane tree and a warp tree join the block's 512 runs
// into f(0, step) and the block folds its q consecutive steps. Runs are
// numbered after `pad` virtual zero runs in front, so every block covers
// exactly q steps and every join is by a fixed length. `base` is 16-byte
// aligned; its first `lead` bytes lie before the data and read as zero.
__global__ void __launch_bounds__(THREADS, 1)
    crc_step_kernel(const uint8_t* __restrict__ base, uint32_t lead, uint64_t pad, uint32_t q,
                    const uint32_t* __restrict__ tabs, uint32_t* __restrict__ partial) {
  extern __shared__ __align__(16) uint32_t sm[];
  uint32_t* rep = sm;
  uint32_t* ops = sm + SLICE_WORDS * 32;  // [0] S_{UNIT/2}, [1 + l] S_{UNIT << l}
  __shared__ uint32_t wv[THREADS / 32];
  const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
  for (uint32_t i = threadIdx.x; i < SLICE_WORDS * 32; i += THREADS) rep[i] = tabs[i >> 5];
  for (uint32_t i = threadIdx.x; i < OPS * OP_WORDS; i += THREADS) ops[i] = tabs[SLICE_WORDS + i];
  __syncthreads();
  const uint32_t* mine = rep + lane;
  constexpr int HALF = UNIT / 32;  // uint4 per half run
  constexpr int IT = HALF / 4;     // iterations per step, 4 uint4 of each half each
  uint4 nxt[8];
  auto fetch = [&](uint32_t g) -> bool {
    const uint32_t st = g / IT, it = g % IT;
    const uint64_t vu = ((uint64_t)blockIdx.x * q + st) * THREADS + threadIdx.x;
    if (vu < pad) return false;
    const uint4* p = reinterpret_cast<const uint4*>(base + (vu - pad) * UNIT) + 4 * it;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      nxt[j] = __ldg(p + j);
      nxt[4 + j] = __ldg(p + HALF + j);
    }
    if (vu == pad && it == 0) {  // run 0: the bytes before the data read as zero
      nxt[0].x = keep_from(nxt[0].x, (int)lead);
      nxt[0].y = keep_from(nxt[0].y, (int)lead - 4);
      nxt[0].z = keep_from(nxt[0].z, (int)lead - 8);
      nxt[0].w = keep_from(nxt[0].w, (int)lead - 12);
    }
    return true;
  };
  const uint32_t total = q * IT;
  bool have_next = fetch(0);
  uint32_t c0 = 0, c1 = 0, acc = 0;
  bool have_run = false;
  for (uint32_t g = 0; g < total; ++g) {
    uint4 cur[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) cur[j] = nxt[j];
    const bool have = have_next;
    have_next = g + 1 < total ? fetch(g + 1) : false;
    if (have) {
      have_run = true;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        c0 = slice4(mine, c0 ^ cur[j].x);
        c1 = slice4(mine, c1 ^ cur[4 + j].x);
        c0 = slice4(mine, c0 ^ cur[j].y);
        c1 = slice4(mine, c1 ^ cur[4 + j].y);
        c0 = slice4(mine, c0 ^ cur[j].z);
        c1 = slice4(mine, c1 ^ cur[4 + j].z);
        c0 = slice4(mine, c0 ^ cur[j].w);
        c1 = slice4(mine, c1 ^ cur[4 + j].w);
      }
    }
    if (g % IT != IT - 1) continue;
    uint32_t c = have_run ? op_apply(ops, c0) ^ c1 : 0u;
    c0 = c1 = 0;
    have_run = false;
#pragma unroll
    for (int l = 0; l < 5; ++l) {  // lane pairs; the right run is UNIT << l bytes
      const uint32_t o = __shfl_down_sync(0xFFFFFFFFu, c, 1u << l);
      if ((lane & ((2u << l) - 1u)) == 0) c = op_apply(ops + (1 + l) * OP_WORDS, c) ^ o;
    }
    if (lane == 0) wv[warp] = c;
    __syncthreads();
    if (warp == 0) {
      c = lane < THREADS / 32 ? wv[lane] : 0u;
#pragma unroll
      for (int l = 0; l < 4; ++l) {  // warp pairs; the right run is 32 * UNIT << l bytes
        const uint32_t o = __shfl_down_sync(0xFFFFFFFFu, c, 1u << l);
        if ((lane & ((2u << l) - 1u)) == 0) c = op_apply(ops + (6 + l) * OP_WORDS, c) ^ o;
      }
      if (lane == 0) acc = op_apply(ops + 10 * OP_WORDS, acc) ^ c;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[blockIdx.x] = acc;
}

struct FinishArgs {
  uint32_t cols[32];  // S_{q * STEP}: joins consecutive blocks
  const uint32_t* partial;
  uint32_t nblk;
  uint32_t tail_len;
  const uint8_t* tail;  // the bytes after the last whole run
  uint32_t fin;         // S_len(~0)
  const uint32_t* tabs;
  uint32_t* out;
};

// One warp: joins the blocks' values in order (one lane per matrix column,
// the product as a XOR reduction), continues the register over the tail and
// writes crc32c = ~(f(0, D) ^ S_len(~0)).
__global__ void __launch_bounds__(32) crc_finish_kernel(const __grid_constant__ FinishArgs a) {
  __shared__ uint32_t t4[SLICE_WORDS];
  const uint32_t lane = threadIdx.x;
  for (uint32_t i = lane; i < SLICE_WORDS; i += 32) t4[i] = a.tabs[i];
  __syncwarp();
  const uint32_t col = a.cols[lane];
  uint32_t acc = 0;
  for (uint32_t b = 0; b < a.nblk; ++b)
    acc = __reduce_xor_sync(0xFFFFFFFFu, ((acc >> lane) & 1u) ? col : 0u) ^ a.partial[b];
  if (lane == 0) {
    const uint8_t* p = a.tail;
    uint32_t n = a.tail_len;
    while (n && (reinterpret_cast<uintptr_t>(p) & 3u)) {
      acc = (acc >> 8) ^ t4[(acc ^ *p++) & 0xFFu];
      --n;
    }
    while (n >= 4) {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(p) ^ acc;
      acc = t4[768 + (w & 0xFFu)] ^ t4[512 + ((w >> 8) & 0xFFu)] ^ t4[256 + ((w >> 16) & 0xFFu)] ^ t4[w >> 24];
      p += 4;
      n -= 4;
    }
    while (n--) acc = (acc >> 8) ^ t4[(acc ^ *p++) & 0xFFu];
    *a.out = ~(acc ^ a.fin);
  }
}

const uint32_t* device_tables(pxc_ctx* ctx) {
  std::lock_guard<std::mutex> lock(ctx->crc_mu);
  if (!ctx->crc_tab) {
    uint32_t* p = nullptr;
    PXC_CUDA(cudaMalloc(&p, DEV_WORDS * 4));
    const cudaError_t e = cudaMemcpy(p, tables().dev.data(), DEV_WORDS * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      cudaFree(p);
      PXC_CUDA(e);
    }
    PXC_CUDA(cudaFuncSetAttribute(crc_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)STEP_SMEM));
    ctx->crc_tab = p;
  }
  return ctx->crc_tab;
}

// Words of scratch one device CRC needs (its block values).
uint32_t scratch_words(const pxc_ctx* ctx) { return (uint32_t)std::max(ctx->sm_count, 1); }

// crc32c of `len` device bytes at `d` into *d_out (device), enqueued on `s`.
// `d` lies in a device allocation whose start is 16-byte aligned (cudaMalloc,
// the caching allocators): the kernel reads from `d` rounded down to 16.
// Returns the kernels launched.
// `tabs` = device_tables(ctx).
int device_crc(pxc_ctx* ctx, const uint32_t* tabs, const void* d, uint64_t len, uint32_t* d_scratch, uint32_t* d_out,
               cudaStream_t s) {
  const Tables& T = tables();
  const uintptr_t addr = reinterpret_cast<uintptr_t>(d);
  const uint32_t lead = (uint32_t)(addr & 15u);
  const uint8_t* base = reinterpret_cast<const uint8_t*>(addr - lead);
  const uint64_t total = lead + len;
  const uint64_t units = total / UNIT;
  uint32_t nblk = 0, q = 0;
  int launches = 0;
  if (units) {
    const uint64_t G = (units + THREADS - 1) / THREADS;
    nblk = (uint32_t)std::min<uint64_t>(G, scratch_words(ctx));
    q = (uint32_t)((G + nblk - 1) / nblk);
    const uint64_t pad = (uint64_t)nblk * q * THREADS - units;
    crc_step_kernel<<<nblk, THREADS, STEP_SMEM, s>>>(base, lead, pad, q, tabs, d_scratch);
    PXC_CUDA(cudaGetLastError());
    ++launches;
  }
  FinishArgs a{};
  const Mat m = T.matrix((uint64_t)q * STEP);
  std::memcpy(a.cols, m.c, sizeof(a.cols));
  a.partial = d_scratch;
  a.nblk = nblk;
  const uint64_t tb = std::max<uint64_t>(lead, units * UNIT);
  a.tail = base + tb;
  a.tail_len = (uint32_t)(total - tb);
  a.fin = T.shift(0xFFFFFFFFu, len);
  a.tabs = tabs;
  a.out = d_out;
  crc_finish_kernel<<<1, 32, 0, s>>>(a);
  PXC_CUDA(cudaGetLastError());
  return launches + 1;
}

}  // namespace crc

// ---------------------------------------------------------------------------
// Codec (codec.rs): little-endian primitives, u32 length prefixes bounded by
// the bytes that remain (codec.rs:296-320), strings checked as UTF-8.
// ---------------------------------------------------------------------------
namespace snap {

constexpr uint8_t MAGIC[8] = {'P', 'R', 'O', 'X', 'S', 'N', 'A', 'P'};
constexpr uint32_t VERSION = 1;
constexpr uint32_t BYTE_ORDER_MARK = 0x01020304u;
constexpr uint64_t HEADER_BYTES = 8 + 4 + 4 + 4 + 8;
constexpr uint8_t KIND_FLAT = 1, KIND_HNSW = 2, KIND_IVFPQ = 3;
constexpr uint64_t CONFIG_BYTES = 4 * 4 + 8 + 4 + 4 + 8 + 1;
constexpr uint64_t REPORT_BYTES = 4 + 8 + 4 + 8 + 4 + 4;

[[noreturn]] void corrupt(const char* structure, const char* fmt, ...) {
  Failure f;
  f.code = PXC_CORRUPTION;
  std::snprintf(f.parameter, sizeof(f.parameter), "%s", structure);
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(f.detail, sizeof(f.detail), fmt, ap);
  va_end(ap);
  throw f;
}

inline uint32_t rd32(const uint8_t* p) {
  uint32_t v;
  std::memcpy(&v, p, 4);
  return v;
}
inline uint64_t rd64(const uint8_t* p) {
  uint64_t v;
  std::memcpy(&v, p, 8);
  return v;
}

// std::str::from_utf8's acceptance: shortest forms only, no surrogates, at
// most U+10FFFF.
bool utf8_valid(const uint8_t* s, uint64_t n) {
  uint64_t i = 0;
  while (i < n) {
    const uint8_t c = s[i];
    if (c < 0x80) {
      ++i;
      continue;
    }
    int len;
    uint32_t lo = 0x80, hi = 0xBF;
    if (c >= 0xC2 && c <= 0xDF) {
      len = 2;
    } else if (c >= 0xE0 && c <= 0xEF) {
      len = 3;
      if (c == 0xE0) lo = 0xA0;
      if (c == 0xED) hi = 0x9F;
    } else if (c >= 0xF0 && c <= 0xF4) {
      len = 4;
      if (c == 0xF0) lo = 0x90;
      if (c == 0xF4) hi = 0x8F;
    } else {
      return false;
    }
    if (n - i < (uint64_t)len) return false;
    if (s[i + 1] < lo || s[i + 1] > hi) return false;
    for (int k = 2; k < len; ++k)
      if (s[i + k] < 0x80 || s[i + k] > 0xBF) return false;
    i += len;
  }
  return true;
}

struct Reader {
  const uint8_t* b;
  uint64_t n;
  const char* structure;
  uint64_t pos = 0;
  Reader(const uint8_t* bytes, uint64_t len, const char* what) : b(bytes), n(len), structure(what) {}
  uint64_t remaining() const { return n - pos; }
  const uint8_t* take(uint64_t count) {
    if (remaining() < count)
      corrupt(structure, "truncated at byte %llu: wanted %llu more, %llu remain", (unsigned long long)pos,
              (unsigned long long)count, (unsigned long long)remaining());
    const uint8_t* p = b + pos;
    pos += count;
    return p;
  }
  uint8_t u8() { return *take(1); }
  uint32_t u32() { return rd32(take(4)); }
  uint64_t u64() { return rd64(take(8)); }
  uint64_t len_prefix(uint64_t element_bytes) {
    const uint32_t length = u32();
    const uint64_t needed = (uint64_t)length * std::max<uint64_t>(element_bytes, 1);
    if (needed > remaining())
      corrupt(structure, "length prefix at byte %llu claims %u elements (%llu bytes) with only %llu left",
              (unsigned long long)(pos - 4), length, (unsigned long long)needed, (unsigned long long)remaining());
    return length;
  }
  void str() {
    const uint64_t len = len_prefix(1);
    const uint8_t* p = take(len);
    if (!utf8_valid(p, len)) corrupt(structure, "field is not UTF-8");
  }
  // A length-prefixed array: (offset of its first element, element count).
  std::pair<uint64_t, uint64_t> array(uint64_t element_bytes) {
    const uint64_t len = len_prefix(element_bytes);
    const uint64_t at = pos;
    take(len * element_bytes);
    return {at, len};
  }
  void metadata() {  // codec.rs:367-392
    const uint64_t count = len_prefix(4);
    for (uint64_t i = 0; i < count; ++i) {
      str();
      const uint8_t tag = u8();
      switch (tag) {
        case 1: str(); break;
        case 2: take(8); break;
        case 3: take(8); break;
        case 4: take(1); break;
        default: corrupt(structure, "metadata value tag %u is not one of 1..=4", tag);
      }
    }
  }
  void expect_end() const {
    if (remaining() != 0)
      corrupt(structure, "%llu trailing bytes after the final field", (unsigned long long)remaining());
  }
};

// Checks the magic, version, reserved word, byte order and length
// (snapshot.rs:331-366); returns the body length. The checksum is the
// caller's.
uint64_t verify_header(const uint8_t* bytes, uint64_t len) {
  if (bytes == nullptr && len) corrupt("snapshot header", "null image");
  if (len < HEADER_BYTES + 4)
    corrupt("snapshot header", "%llu bytes is shorter than the %llu-byte header plus checksum",
            (unsigned long long)len, (unsigned long long)HEADER_BYTES);
  if (std::memcmp(bytes, MAGIC, 8) != 0) corrupt("snapshot header", "expected magic \"PROXSNAP\"");
  const uint32_t version = rd32(bytes + 8);
  if (version != VERSION) corrupt("snapshot header", "format version %u, this build reads %u", version, VERSION);
  const uint32_t reserved = rd32(bytes + 16);
  if (reserved != 0) corrupt("snapshot header", "reserved word is 0x%08x, not zero", reserved);
  const uint32_t order = rd32(bytes + 12);
  if (order != BYTE_ORDER_MARK)
    corrupt("snapshot header",
            "byte-order mark 0x%08x means the file was written on a machine of the opposite endianness", order);
  const uint64_t body_len = rd64(bytes + 20);
  if (len - HEADER_BYTES - 4 != body_len)
    corrupt("snapshot", "header claims a %llu-byte body, file holds %llu", (unsigned long long)body_len,
            (unsigned long long)(len - HEADER_BYTES - 4));
  return body_len;
}

uint32_t recorded_crc(const uint8_t* bytes, uint64_t body_len) { return rd32(bytes + HEADER_BYTES + body_len); }

[[noreturn]] void checksum_mismatch(uint32_t actual, uint32_t expected) {
  corrupt("snapshot", "checksum 0x%08x does not match the recorded 0x%08x", actual, expected);
}

int32_t metric_from_tag(uint8_t tag) {  // codec.rs:414-426
  switch (tag) {
    case 1: return PXC_EUCLIDEAN;
    case 2: return PXC_COSINE;
    case 3: return PXC_INNER_PRODUCT;
    case 4: return PXC_MANHATTAN;
    default: corrupt("snapshot body", "metric tag %u is not one of 1..=4", tag);
  }
}
uint8_t metric_tag(int32_t metric) {
  switch (metric) {
    case PXC_EUCLIDEAN: return 1;
    case PXC_COSINE: return 2;
    case PXC_INNER_PRODUCT: return 3;
    default: return 4;
  }
}

// Where everything of an IVF-PQ body is (offsets from the body start).
struct IvfPqBody {
  uint32_t dim = 0;
  int32_t metric = 0;
  uint8_t kind = 0;
  pxc_ivfpq_config config{};
  uint64_t ids_at = 0, nslots = 0;  // first id record
  uint64_t meta_at = 0, meta_bytes = 0, meta_count = 0;
  std::pair<uint64_t, uint64_t> vectors{}, codes{}, list_of{}, centroids{}, codebooks{};
  bool has_report = false;
  pxc_ivfpq_report report{};
  uint64_t trailing = 0;
};

// Reads the space, the kind and, for an IVF-PQ body, every section
// (snapshot.rs:204-262, 481-516). Stops after the space and kind of another
// kind of index.
IvfPqBody parse_body(const uint8_t* body, uint64_t n) {
  IvfPqBody r;
  Reader rd(body, n, "snapshot body");
  r.dim = rd.u32();
  r.metric = metric_from_tag(rd.u8());
  if (r.dim < 1 || r.dim > (1u << 20)) {
    Failure f = make_failure(PXC_CONFIGURATION, r.dim, 0, "dim", "%s",
                             r.dim < 1 ? "must be at least 1; a 0-dimensional space makes all distances equal"
                                       : "exceeds the 1048576 dimension ceiling");
    throw f;
  }
  r.kind = rd.u8();
  if (r.kind < KIND_FLAT || r.kind > KIND_IVFPQ) corrupt("snapshot body", "index kind %u is not one of 1..=3", r.kind);
  if (r.kind != KIND_IVFPQ) return r;
  auto& c = r.config;
  c.nlist = rd.u32();
  c.subspaces = rd.u32();
  c.nprobe = rd.u32();
  c.rerank = rd.u32();
  c.seed = rd.u64();
  c.max_iterations = rd.u32();
  c.training_sample = rd.u32();
  c.train_threshold = rd.u64();
  c.retain_vectors = rd.u8() != 0 ? 1u : 0u;
  r.nslots = rd.len_prefix(9);
  r.ids_at = rd.pos;
  rd.take(r.nslots * 9);
  r.meta_at = rd.pos;
  r.meta_count = rd.len_prefix(4);
  for (uint64_t i = 0; i < r.meta_count; ++i) rd.metadata();
  r.meta_bytes = rd.pos - r.meta_at;
  r.vectors = rd.array(4);
  r.codes = rd.array(1);
  r.list_of = rd.array(4);
  r.centroids = rd.array(4);
  r.codebooks = rd.array(4);
  if (rd.u8() != 0) {
    r.has_report = true;
    r.report.sampled = rd.u32();
    std::memcpy(&r.report.coarse_inertia, rd.take(8), 8);
    r.report.coarse_iterations = rd.u32();
    std::memcpy(&r.report.residual_inertia, rd.take(8), 8);
    r.report.populated_lists = rd.u32();
    r.report.largest_list = rd.u32();
  }
  r.trailing = rd.remaining();
  return r;
}


const char* kind_name(uint8_t kind) { return kind == KIND_FLAT ? "flat" : kind == KIND_HNSW ? "hnsw" : "ivfpq"; }

// IvfPqIndex::new (ivfpq.rs:481-491), IvfPqConfig::validate (:259-302), the
// length checks of from_parts (:631-663), ProductQuantizer::from_parts
// (product.rs:463-503), then this build's device limits.
void validate_parts(const IvfPqBody& r) {
  const auto& c = r.config;
  if (r.metric != PXC_EUCLIDEAN && r.metric != PXC_COSINE)
    throw make_failure(PXC_CONFIGURATION, (uint64_t)r.metric, 0, "metric", "%s",
                       "IVF-PQ supports euclidean and cosine only");
  if (c.nlist == 0) throw make_failure(PXC_CONFIGURATION, 0, 0, "nlist", "%s", "must be at least 1");
  if (c.subspaces == 0 || c.subspaces > r.dim)
    throw make_failure(PXC_CONFIGURATION, c.subspaces, 0, "subspaces", "%s",
                       "must be between 1 and the space dimension");
  if (c.nprobe == 0 || c.nprobe > c.nlist)
    throw make_failure(PXC_CONFIGURATION, c.nprobe, 0, "nprobe", "%s", "must be between 1 and nlist");
  if (c.max_iterations == 0) throw make_failure(PXC_CONFIGURATION, 0, 0, "max_iterations", "%s", "must be at least 1");
  if (c.training_sample == 0)
    throw make_failure(PXC_CONFIGURATION, 0, 0, "training_sample", "%s", "must be at least 1");
  if (c.rerank > 0 && !c.retain_vectors)
    throw make_failure(PXC_CONFIGURATION, c.rerank, 0, "rerank", "%s",
                       "requires retain_vectors, because reranking is against the exact vectors");
  const uint64_t n = r.nslots, dim = r.dim, m = c.subspaces;
  auto check = [](const char* what, uint64_t actual, uint64_t expected) {
    if (actual != expected)
      corrupt("ivfpq index", "%s holds %llu entries, expected %llu", what, (unsigned long long)actual,
              (unsigned long long)expected);
  };
  check("metadata", r.meta_count, n);
  if (r.vectors.second) check("vectors", r.vectors.second, n * dim);
  if (r.codes.second) {
    check("codes", r.codes.second, n * m);
    check("list assignments", r.list_of.second, n);
  }
  if (r.centroids.second) {
    if (r.centroids.second % dim)
      corrupt("ivfpq centroids", "%llu floats is not a multiple of dimension %llu",
              (unsigned long long)r.centroids.second, (unsigned long long)dim);
    if (r.codebooks.second != 256 * dim)
      corrupt("product quantizer", "%llu codebook floats for %llu subspaces of dimension %llu, expected %llu",
              (unsigned long long)r.codebooks.second, (unsigned long long)m, (unsigned long long)dim,
              (unsigned long long)(256 * dim));
  }
  if (!r.codes.second && r.list_of.second > n)
    corrupt("ivfpq index", "list assignments hold %llu entries for %llu slots", (unsigned long long)r.list_of.second,
            (unsigned long long)n);
  PXC_CONFIG(r.dim <= ivf::MAX_DIM, "dim", r.dim, "the device IVF-PQ supports 1 <= dim <= 1024");
  PXC_CONFIG(m <= ivf::MAX_M, "subspaces", m, "the device IVF-PQ supports at most 64 subspaces");
  PXC_CONFIG(n < 0xFFFFFFFFull, "nslots", n, "the device IVF-PQ supports fewer than 2^32 slots");
}

uint32_t lists_of(const IvfPqBody& r) {
  return r.centroids.second ? (uint32_t)(r.centroids.second / r.dim) : r.config.nlist;
}

// The from_parts checks a host pass can make over assignments that do not go
// to the device (list_of without codes), and the duplicate-id check of a
// host-only read.
void check_ids_host(const IvfPqBody& r, const uint8_t* body) {
  const uint8_t* idp = body + r.ids_at;
  std::vector<std::pair<uint64_t, uint64_t>> seen;  // (id, slot) of present slots
  seen.reserve(r.nslots);
  for (uint64_t i = 0; i < r.nslots; ++i)
    if (idp[9 * i]) seen.emplace_back(rd64(idp + 9 * i + 1), i);
  std::sort(seen.begin(), seen.end());
  uint64_t dup = UINT64_MAX, dup_id = 0;
  for (size_t k = 1; k < seen.size(); ++k)
    if (seen[k].first == seen[k - 1].first && seen[k].second < dup) {
      dup = seen[k].second;
      dup_id = seen[k].first;
    }
  if (dup != UINT64_MAX) corrupt("ivfpq index", "id %llu appears at two slots", (unsigned long long)dup_id);
}

void check_lists_host(const IvfPqBody& r, const uint8_t* body) {
  const uint32_t lists = lists_of(r);
  const uint8_t* idp = body + r.ids_at;
  const uint8_t* lp = body + r.list_of.first;
  for (uint64_t i = 0; i < r.list_of.second; ++i) {
    const uint32_t l = rd32(lp + 4 * i);
    if (l == ivf::UNASSIGNED || !idp[9 * i]) continue;
    if (l >= lists) corrupt("ivfpq index", "slot %llu names list %u of %u", (unsigned long long)i, l, lists);
  }
}

void fill_info(const IvfPqBody& r, uint64_t body_len, uint64_t live, pxc_snapshot_info* info) {
  if (!info) return;
  std::memset(info, 0, sizeof(*info));
  info->format_version = VERSION;
  info->kind = r.kind;
  info->dim = r.dim;
  info->metric = r.metric;
  info->body_bytes = body_len;
  info->nslots = r.nslots;
  info->live = live;
  if (r.kind != KIND_IVFPQ) return;
  info->metadata_offset = HEADER_BYTES + r.meta_at;
  info->metadata_bytes = r.meta_bytes;
  info->config = r.config;
  info->trained = r.centroids.second ? 1u : 0u;
  info->lists = lists_of(r);
  info->has_vectors = r.vectors.second ? 1u : 0u;
  info->has_report = r.has_report ? 1u : 0u;
  if (r.has_report) info->report = r.report;
}

// The store's id table of a flat or HNSW body, for peek (snapshot.rs:383-405).
void store_ids(const uint8_t* body, uint64_t n, IvfPqBody& r) {
  Reader rd(body, n, "snapshot body");
  rd.take(4 + 1 + 1);
  if (r.kind == KIND_HNSW) rd.take(4 * 4 + 8 + 4 + 1 + 1);
  r.nslots = rd.len_prefix(9);
  r.ids_at = rd.pos;
}

uint64_t count_live(const IvfPqBody& r, const uint8_t* body) {
  uint64_t live = 0;
  for (uint64_t i = 0; i < r.nslots; ++i) live += body[r.ids_at + 9 * i] != 0;
  return live;
}

struct Writer {
  uint8_t* p;
  uint64_t pos = 0;
  explicit Writer(uint8_t* out) : p(out) {}
  void u8(uint8_t v) { p[pos++] = v; }
  void u32(uint32_t v) {
    std::memcpy(p + pos, &v, 4);
    pos += 4;
  }
  void u64(uint64_t v) {
    std::memcpy(p + pos, &v, 8);
    pos += 8;
  }
  void f64(double v) {
    std::memcpy(p + pos, &v, 8);
    pos += 8;
  }
  void raw(const void* src, uint64_t n) {
    if (n) std::memcpy(p + pos, src, n);
    pos += n;
  }
};

inline uint32_t saturate(uint64_t v) { return v > 0xFFFFFFFFull ? 0xFFFFFFFFu : (uint32_t)v; }

}  // namespace snap
}  // namespace pxc

using namespace pxc;

namespace {

__global__ void snapshot_list_keys_kernel(const uint32_t* __restrict__ list_of, const uint8_t* __restrict__ live,
                                          uint64_t n, uint32_t nlist, uint32_t* __restrict__ keys,
                                          uint32_t* __restrict__ bad) {
  const uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t l = list_of[i];
  uint32_t key = ivf::UNASSIGNED;
  if (live[i] && l != ivf::UNASSIGNED) {
    if (l < nlist)
      key = l;
    else
      atomicMin(bad, (uint32_t)i);
  }
  keys[i] = key;
}

// A body piece either on the host (checksummed there) or in a device array
// (checksummed on the device).
struct Piece {
  uint64_t bytes;
  int device;  // index of the device CRC, -1 for host
  const uint8_t* host;
};

uint32_t join_pieces(const std::vector<Piece>& pieces, const uint32_t* dev_crc) {
  uint32_t acc = 0;
  for (const Piece& pc : pieces) {
    const uint32_t c = pc.device >= 0 ? dev_crc[pc.device] : crc::append(0, pc.host, pc.bytes);
    acc = crc::combine(acc, c, pc.bytes);
  }
  return acc;
}

}  // namespace

extern "C" {

uint32_t pxc_crc32c_append(uint32_t crc, const void* bytes, uint64_t len) {
  if (!bytes || !len) return crc;
  return crc::append(crc, bytes, len);
}

uint32_t pxc_crc32c_combine(uint32_t crc_a, uint32_t crc_b, uint64_t len_b) { return crc::combine(crc_a, crc_b, len_b); }

pxc_status pxc_crc32c_device(pxc_ctx* ctx, const void* d_bytes, uint64_t len, uint32_t* out, void* stream,
                             pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(out != nullptr, "out", 0, "null output");
    PXC_CONFIG(d_bytes != nullptr || len == 0, "d_bytes", 0, "null input");
    DeviceGuard g(ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
    const uint32_t sw = crc::scratch_words(ctx);
    const uint32_t* tabs = crc::device_tables(ctx);
    std::lock_guard<std::mutex> lock(ctx->crc_mu);  // the context's scratch and result word
    if (!ctx->crc_scratch) PXC_CUDA(cudaMalloc(&ctx->crc_scratch, ((size_t)sw + 1) * 4));
    if (!ctx->crc_host) PXC_CUDA(cudaMallocHost(&ctx->crc_host, 4));
    ctx->launches += crc::device_crc(ctx, tabs, len ? d_bytes : ctx->crc_scratch, len, ctx->crc_scratch,
                                     ctx->crc_scratch + sw, s);
    PXC_CUDA(cudaMemcpyAsync(ctx->crc_host, ctx->crc_scratch + sw, 4, cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    *out = *ctx->crc_host;
  });
}

pxc_status pxc_snapshot_peek(const uint8_t* bytes, uint64_t len, pxc_snapshot_info* info, pxc_error* err) {
  return guarded(err, [&] {
    const uint64_t body_len = snap::verify_header(bytes, len);
    const uint8_t* body = bytes + snap::HEADER_BYTES;
    const uint32_t actual = crc::append(0, body, body_len), expected = snap::recorded_crc(bytes, body_len);
    if (actual != expected) snap::checksum_mismatch(actual, expected);
    snap::IvfPqBody r = snap::parse_body(body, body_len);
    if (r.kind == snap::KIND_IVFPQ) {
      snap::validate_parts(r);
      snap::check_ids_host(r, body);
      snap::check_lists_host(r, body);
      if (r.trailing)
        snap::corrupt("snapshot body", "%llu trailing bytes after the final field", (unsigned long long)r.trailing);
    } else {
      snap::store_ids(body, body_len, r);
    }
    snap::fill_info(r, body_len, snap::count_live(r, body), info);
  });
}

pxc_status pxc_ivfpq_snapshot_load(pxc_ctx* ctx, const uint8_t* bytes, uint64_t len, pxc_ivfpq** out,
                                   pxc_snapshot_info* info, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr, "ctx", 0, "null context");
    PXC_CONFIG(out != nullptr, "out", 0, "output handle pointer is null");
    *out = nullptr;
    const uint64_t body_len = snap::verify_header(bytes, len);
    const uint8_t* body = bytes + snap::HEADER_BYTES;
    const uint32_t expected = snap::recorded_crc(bytes, body_len);
    snap::IvfPqBody r;
    try {
      r = snap::parse_body(body, body_len);
      if (r.kind != snap::KIND_IVFPQ)
        throw make_failure(PXC_CONFIGURATION, r.kind, 0, "kind", "the snapshot holds a %s index, not IVF-PQ",
                           snap::kind_name(r.kind));
      snap::validate_parts(r);
      if (!r.codes.second) snap::check_lists_host(r, body);  // assignments that stay on the host
    } catch (const Failure&) {
      // the reference verifies the checksum before it decodes anything
      const uint32_t actual = crc::append(0, body, body_len);
      if (actual != expected) snap::checksum_mismatch(actual, expected);
      throw;
    }
    DeviceGuard g(ctx->device);
    cudaStream_t s = ctx->stream;
    const uint32_t dim = r.dim, m = r.config.subspaces, lists = snap::lists_of(r);
    const uint64_t n = r.nslots;
    pxc_ivfpq* raw = nullptr;
    {
      pxc_error e2{};
      const pxc_status st = pxc_ivfpq_create(ctx, dim, r.metric, lists, m, &raw, &e2);
      if (st != PXC_OK) throw make_failure(st, e2.a, e2.b, e2.parameter, "%s", e2.detail);
    }
    std::unique_ptr<pxc_ivfpq, void (*)(pxc_ivfpq*)> hold(raw, pxc_ivfpq_destroy);
    pxc_ivfpq* h = raw;
    std::lock_guard<std::mutex> lock(h->mu);
    // ids: the host keeps them (tombstones as id 0), the device ranks them
    h->nslots = n;
    h->h_ids.resize(n);
    h->h_live.resize(n);
    std::vector<uint32_t> live_slots;
    std::vector<uint64_t> live_ids;
    live_slots.reserve(n);
    live_ids.reserve(n);
    const uint8_t* idp = body + r.ids_at;
    for (uint64_t i = 0; i < n; ++i) {
      const bool present = idp[9 * i] != 0;
      const uint64_t id = snap::rd64(idp + 9 * i + 1);
      h->h_ids[i] = present ? id : 0;
      h->h_live[i] = present ? 1 : 0;
      if (present) {
        live_slots.push_back((uint32_t)i);
        live_ids.push_back(id);
      }
    }
    const uint64_t nlive = live_slots.size();
    const uint32_t sw = crc::scratch_words(ctx);
    const uint32_t* tabs = crc::device_tables(ctx);
    DBuf<uint32_t> scratch, d_live_slots, keys;
    DBuf<uint64_t> d_live_ids;
    scratch.reserve(5 * (size_t)sw + 8);
    uint32_t* d_crc = scratch.p + 5 * (size_t)sw;  // [0..5) array CRCs, [5] duplicate slot, [6] bad list slot
    PXC_CUDA(cudaMemsetAsync(d_crc, 0xFF, 8 * 4, s));
    h->ids.reserve(std::max<uint64_t>(1, n));
    h->live.reserve(std::max<uint64_t>(1, n));
    d_live_slots.reserve(std::max<uint64_t>(1, nlive));
    d_live_ids.reserve(std::max<uint64_t>(1, nlive));
    hostcopy::to_device(ctx, h->ids.p, h->h_ids.data(), n * 8, s);
    hostcopy::to_device(ctx, h->live.p, h->h_live.data(), n, s);
    hostcopy::to_device(ctx, d_live_slots.p, live_slots.data(), nlive * 4, s);
    hostcopy::to_device(ctx, d_live_ids.p, live_ids.data(), nlive * 8, s);
    // the arrays: one copy each from the image, then their CRC on the device
    std::vector<Piece> pieces;
    uint64_t at = 0;
    int next = 0;
    auto array = [&](const std::pair<uint64_t, uint64_t>& sec, uint64_t elem, void* dst) {
      pieces.push_back({sec.first - at, -1, body + at});
      const uint64_t nb = sec.second * elem;
      at = sec.first + nb;
      if (!nb) return;
      hostcopy::to_device(ctx, dst, body + sec.first, nb, s);
      ctx->launches += crc::device_crc(ctx, tabs, dst, nb, scratch.p + (size_t)next * sw, d_crc + next, s);
      pieces.push_back({nb, next++, nullptr});
    };
    if (r.vectors.second) h->vectors.reserve(r.vectors.second);
    if (r.codes.second) {
      h->codes.reserve(std::max<uint64_t>(16, r.codes.second));
      h->list_of.reserve(std::max<uint64_t>(1, r.list_of.second));
    }
    if (r.centroids.second) {
      h->centroids.reserve(r.centroids.second);
      h->codebooks.reserve(r.codebooks.second);
    }
    array(r.vectors, 4, h->vectors.p);
    array(r.codes, 1, h->codes.p);
    if (r.codes.second) array(r.list_of, 4, h->list_of.p);  // (without codes they stay in the host piece)
    if (r.centroids.second) {
      array(r.centroids, 4, h->centroids.p);
      array(r.codebooks, 4, h->codebooks.p);
    }
    pieces.push_back({body_len - at, -1, body + at});
    // ranks, then the lists
    ivf::rank_ids_device(h, d_live_slots.p, d_live_ids.p, nlive, d_crc + 5, s);
    if (r.codes.second && n) {
      keys.reserve(n);
      snapshot_list_keys_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(h->list_of.p, h->live.p, n, lists, keys.p,
                                                                            d_crc + 6);
      PXC_CUDA(cudaGetLastError());
      ctx->launches += 1;
      ivf::build_lists_device(h, keys.p, s);
    }
    uint32_t hc[8];
    PXC_CUDA(cudaMemcpyAsync(hc, d_crc, sizeof(hc), cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    const uint32_t actual = join_pieces(pieces, hc);
    if (actual != expected) snap::checksum_mismatch(actual, expected);
    if (hc[5] != 0xFFFFFFFFu)
      snap::corrupt("ivfpq index", "id %llu appears at two slots", (unsigned long long)h->h_ids[hc[5]]);
    if (hc[6] != 0xFFFFFFFFu)
      snap::corrupt("ivfpq index", "slot %u names list %u of %u", hc[6],
                    snap::rd32(body + r.list_of.first + 4 * (uint64_t)hc[6]), lists);
    if (r.trailing)
      snap::corrupt("snapshot body", "%llu trailing bytes after the final field", (unsigned long long)r.trailing);
    h->have_parts = r.centroids.second != 0;
    h->have_vectors = r.vectors.second != 0;
    h->u8_state = 0;
    snap::fill_info(r, body_len, nlive, info);
    *out = hold.release();
  });
}

pxc_status pxc_ivfpq_snapshot_save(pxc_ivfpq* h, const pxc_ivfpq_config* config, const pxc_ivfpq_report* report,
                                   const uint8_t* metadata, uint64_t metadata_bytes, uint8_t* out, uint64_t capacity,
                                   uint64_t* out_len, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(h != nullptr, "h", 0, "null handle");
    PXC_CONFIG(config != nullptr, "config", 0, "null config");
    PXC_CONFIG(out_len != nullptr, "out_len", 0, "null output length");
    PXC_CONFIG(config->subspaces == h->m, "subspaces", config->subspaces, "differs from the index's subspace count");
    std::lock_guard<std::mutex> lock(h->mu);
    pxc_ctx* ctx = h->ctx;
    DeviceGuard g(ctx->device);
    cudaStream_t s = ctx->stream;
    ivf::handoff_drain(h);
    const uint64_t n = h->nslots, dim = h->dim, m = h->m;
    if (metadata) {
      snap::Reader rd(metadata, metadata_bytes, "metadata");
      try {
        const uint64_t count = rd.len_prefix(4);
        if (count != n)
          throw make_failure(PXC_CONFIGURATION, count, n, "metadata", "the section holds %llu entries for %llu slots",
                             (unsigned long long)count, (unsigned long long)n);
        for (uint64_t i = 0; i < count; ++i) rd.metadata();
        rd.expect_end();
      } catch (Failure& f) {
        f.code = PXC_CONFIGURATION;
        throw;
      }
    }
    const uint64_t meta = metadata ? metadata_bytes : 4 + 4 * n;
    const uint64_t nvec = h->have_vectors ? n * dim : 0;
    const uint64_t ncode = h->have_lists ? n * m : 0, nlo = h->have_lists ? n : 0;
    const uint64_t ncen = h->have_parts ? (uint64_t)h->nlist * dim : 0, nbook = h->have_parts ? 256 * dim : 0;
    for (uint64_t c : {n, nvec, ncode, ncen, nbook})
      if (c > 0xFFFFFFFFull)
        throw make_failure(PXC_CAPACITY, 0xFFFFFFFFull, c, "snapshot", "%s",
                           "an array of more than 2^32 - 1 elements does not fit the format's u32 length prefix");
    const uint64_t head = 4 + 1 + 1 + snap::CONFIG_BYTES + 4 + 9 * n + meta;
    const uint64_t body_len = head + 4 + nvec * 4 + 4 + ncode + 4 + nlo * 4 + 4 + ncen * 4 + 4 + nbook * 4 + 1 +
                              (report ? snap::REPORT_BYTES : 0);
    const uint64_t total = snap::HEADER_BYTES + body_len + 4;
    *out_len = total;
    if (!out) return;
    if (capacity < total)
      throw make_failure(PXC_CAPACITY, total, capacity, "capacity", "the snapshot needs %llu bytes",
                         (unsigned long long)total);
    snap::Writer w(out);
    w.raw(snap::MAGIC, 8);
    w.u32(snap::VERSION);
    w.u32(snap::BYTE_ORDER_MARK);
    w.u32(0);
    w.u64(body_len);
    uint8_t* body = out + snap::HEADER_BYTES;
    w.u32(h->dim);
    w.u8(snap::metric_tag(h->metric));
    w.u8(snap::KIND_IVFPQ);
    w.u32(config->nlist);
    w.u32(config->subspaces);
    w.u32(config->nprobe);
    w.u32(config->rerank);
    w.u64(config->seed);
    w.u32(config->max_iterations);
    w.u32(config->training_sample);
    w.u64(config->train_threshold);
    w.u8(config->retain_vectors ? 1 : 0);
    w.u32((uint32_t)n);
    for (uint64_t i = 0; i < n; ++i) {
      const bool live = h->h_live[i] != 0;
      w.u8(live ? 1 : 0);
      w.u64(live ? h->h_ids[i] : 0);
    }
    if (metadata) {
      w.raw(metadata, metadata_bytes);
    } else {
      w.u32((uint32_t)n);
      std::memset(out + w.pos, 0, 4 * n);
      w.pos += 4 * n;
    }
    const uint32_t sw = crc::scratch_words(ctx);
    const uint32_t* tabs = crc::device_tables(ctx);
    DBuf<uint32_t> scratch;
    scratch.reserve(5 * (size_t)sw + 8);
    uint32_t* d_crc = scratch.p + 5 * (size_t)sw;
    std::vector<Piece> pieces;
    uint64_t mark = 0;  // start of the current host piece, from the body start
    int next = 0;
    auto array = [&](const void* src, uint64_t count, uint64_t elem) {
      w.u32((uint32_t)count);
      const uint64_t nb = count * elem;
      const uint64_t at = w.pos - snap::HEADER_BYTES;
      pieces.push_back({at - mark, -1, body + mark});
      if (nb) {
        ctx->launches += crc::device_crc(ctx, tabs, src, nb, scratch.p + (size_t)next * sw, d_crc + next, s);
        hostcopy::to_host(ctx, out + w.pos, src, nb, s);
        pieces.push_back({nb, next++, nullptr});
      }
      w.pos += nb;
      mark = at + nb;
    };
    array(h->vectors.p, nvec, 4);
    array(h->codes.p, ncode, 1);
    array(h->list_of.p, nlo, 4);
    array(h->centroids.p, ncen, 4);
    array(h->codebooks.p, nbook, 4);
    if (report) {
      w.u8(1);
      w.u32(snap::saturate(report->sampled));
      w.f64(report->coarse_inertia);
      w.u32(snap::saturate(report->coarse_iterations));
      w.f64(report->residual_inertia);
      w.u32(snap::saturate(report->populated_lists));
      w.u32(snap::saturate(report->largest_list));
    } else {
      w.u8(0);
    }
    pieces.push_back({body_len - mark, -1, body + mark});
    uint32_t hc[8] = {0};
    PXC_CUDA(cudaMemcpyAsync(hc, d_crc, sizeof(hc), cudaMemcpyDeviceToHost, s));
    PXC_CUDA(cudaStreamSynchronize(s));
    w.u32(join_pieces(pieces, hc));
    if (w.pos != total)
      throw make_failure(PXC_INTERNAL, w.pos, total, "snapshot", "%s", "the writer's length disagrees with its plan");
  });
}

}  // extern "C"
