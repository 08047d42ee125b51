// fixtures.cpp — deterministic synthetic workloads (host, C++17).
//
// The reference generates its benchmark corpora (crates/proxima-cli/src/fixture.rs,
// examples/quickstart.rs, crates/proxima-quantize/tests/recall.rs:57-98); no
// external dataset is involved. These generators produce the same shapes and
// value distributions. They are counter-based (element i of a stream is a pure
// function of the seed and i), so any thread count and any slice of rows give
// identical bytes. Normal draws are Irwin-Hall sums of integer uniforms, pure
// integer and IEEE double arithmetic with no libm call, so the values are the
// same on every machine. Build with -ffp-contract=off.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

inline uint64_t mix64(uint64_t z) {  // splitmix64 finaliser (Steele, Lea, Flood 2014)
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
// Element `i` of the splitmix64 stream started at `seed`.
inline uint64_t stream_at(uint64_t seed, uint64_t i) {
  return mix64(seed + 0x9E3779B97F4A7C15ull * (i + 1));
}
inline double unit53(uint64_t x) { return static_cast<double>(x >> 11) * 0x1.0p-53; }
// Approximately N(0,1): Irwin-Hall sum of four 24-bit uniforms, centred and
// scaled to unit variance. The sum is exact; one double multiply rounds.
inline double normal4(uint64_t seed, uint64_t i) {
  int64_t s = 0;
  for (int j = 0; j < 4; ++j) s += static_cast<int64_t>(stream_at(seed, 4 * i + j) >> 40);
  double z = static_cast<double>(s - (int64_t(1) << 25)) * 0x1.0p-24;  // var 1/3
  return z * 1.7320508075688772;
}

template <class F>
void parallel_rows(uint64_t n, int threads, F fn) {
  if (threads <= 1 || n < 1024) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    uint64_t b = n * t / threads, e = n * (t + 1) / threads;
    pool.emplace_back([=] { fn(b, e); });
  }
  for (auto& th : pool) th.join();
}

// distance.rs:508-517 restated for the generator (8-lane dot, sqrt, 1/n, *).
void normalize8(float* v, uint64_t dim) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  uint64_t full = dim / 8 * 8;
  for (uint64_t i = 0; i < full; i += 8)
    for (int l = 0; l < 8; ++l) acc[l] += v[i + l] * v[i + l];
  float tail = 0.0f;
  for (uint64_t i = full; i < dim; ++i) tail += v[i] * v[i];
  float a = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  float b = (acc[4] + acc[5]) + (acc[6] + acc[7]);
  float n = std::sqrt((a + b) + tail);
  if (n > 0.0f && std::isfinite(n)) {
    float inv = 1.0f / n;
    for (uint64_t i = 0; i < dim; ++i) v[i] *= inv;
  }
}

}  // namespace

extern "C" {

// examples/quickstart.rs:25-36 — v[id][d] = sin(cluster*0.7 + d*0.11) + id*0.00002*d,
// all in f32, sin from the platform libm (sinf), as Rust's f32::sin.
void pxf_quickstart(uint64_t count, uint64_t dim, float* out) {
  for (uint64_t id = 0; id < count; ++id) {
    float cluster = static_cast<float>(id % 50);
    for (uint64_t d = 0; d < dim; ++d) {
      float arg = cluster * 0.7f + static_cast<float>(d) * 0.11f;
      float drift = static_cast<float>(id) * 0.00002f * static_cast<float>(d);
      out[id * dim + d] = sinf(arg) + drift;
    }
  }
}

// crates/proxima-quantize/tests/recall.rs:57-98 — splitmix64 uniforms
// (z >> 40) / 4096 - 1, "normal" = sum of six / 2, 32 centres * 3.0, points
// centre + normal * 0.6, point i in cluster i % 32.
void pxf_splitmix_corpus(uint64_t count, uint64_t dim, uint64_t seed, float* out) {
  uint64_t state = seed;
  auto next_f32 = [&]() -> float {
    state += 0x9E3779B97F4A7C15ull;
    uint64_t z = mix64(state);
    return static_cast<float>(z >> 40) / 4096.0f - 1.0f;
  };
  auto next_normal = [&]() -> float {
    float s = 0.0f;
    for (int i = 0; i < 6; ++i) s += next_f32();
    return s / 2.0f;
  };
  std::vector<float> centres(32 * dim);
  for (uint64_t c = 0; c < 32; ++c)
    for (uint64_t d = 0; d < dim; ++d) centres[c * dim + d] = next_normal() * 3.0f;
  for (uint64_t i = 0; i < count; ++i) {
    const float* c = centres.data() + (i % 32) * dim;
    for (uint64_t d = 0; d < dim; ++d) out[i * dim + d] = c[d] + next_normal() * 0.6f;
  }
}

// Integer-valued Gaussian blobs in [0,255]^dim: centres uniform in
// [0,255]^dim from `centre_seed`; row i belongs to blob i % nblobs and is
// clip(round(centre + sigma * N(0,1)), 0, 255) with noise from `noise_seed`,
// stored as f32. Rows [row_begin, row_begin + n) of the stream are produced.
void pxf_blobs_u8(uint64_t row_begin, uint64_t n, uint64_t dim, uint64_t nblobs,
                  uint64_t centre_seed, uint64_t noise_seed, double sigma, float* out,
                  int threads) {
  parallel_rows(n, threads, [&](uint64_t b, uint64_t e) {
    for (uint64_t r = b; r < e; ++r) {
      uint64_t i = row_begin + r;
      uint64_t blob = i % nblobs;
      for (uint64_t d = 0; d < dim; ++d) {
        double c = 255.0 * unit53(stream_at(centre_seed, blob * dim + d));
        double v = c + sigma * normal4(noise_seed, i * dim + d);
        double rv = std::floor(v + 0.5);
        rv = rv < 0.0 ? 0.0 : (rv > 255.0 ? 255.0 : rv);
        out[r * dim + d] = static_cast<float>(rv);
      }
    }
  });
}

// Rows row_first, row_first + stride, ... (n of them) of pxf_blobs_u8's
// stream: a stride sample without generating the rows in between.
void pxf_blobs_u8_strided(uint64_t row_first, uint64_t stride, uint64_t n, uint64_t dim, uint64_t nblobs,
                          uint64_t centre_seed, uint64_t noise_seed, double sigma, float* out, int threads) {
  parallel_rows(n, threads, [&](uint64_t b, uint64_t e) {
    for (uint64_t r = b; r < e; ++r) pxf_blobs_u8(row_first + r * stride, 1, dim, nblobs, centre_seed, noise_seed,
                                                   sigma, out + r * dim, 1);
  });
}

// The same blobs without rounding or clipping: real-valued rows (the
// non-integer counterpart of C2 for the f16 tensor-core screen).
void pxf_blobs_f32(uint64_t row_begin, uint64_t n, uint64_t dim, uint64_t nblobs,
                   uint64_t centre_seed, uint64_t noise_seed, double sigma, float* out,
                   int threads) {
  parallel_rows(n, threads, [&](uint64_t b, uint64_t e) {
    for (uint64_t r = b; r < e; ++r) {
      uint64_t i = row_begin + r;
      uint64_t blob = i % nblobs;
      for (uint64_t d = 0; d < dim; ++d) {
        double c = 255.0 * unit53(stream_at(centre_seed, blob * dim + d));
        out[r * dim + d] = static_cast<float>(c + sigma * normal4(noise_seed, i * dim + d));
      }
    }
  });
}

// Unit-sphere blobs: centre = normalize(N(0,1)^dim) from `centre_seed`; row i
// of blob i % nblobs is normalize(centre + sigma * N(0,1)) from `noise_seed`.
void pxf_sphere_blobs(uint64_t row_begin, uint64_t n, uint64_t dim, uint64_t nblobs,
                      uint64_t centre_seed, uint64_t noise_seed, double sigma, float* out,
                      int threads) {
  parallel_rows(n, threads, [&](uint64_t b, uint64_t e) {
    std::vector<float> c(dim);
    for (uint64_t r = b; r < e; ++r) {
      uint64_t i = row_begin + r;
      uint64_t blob = i % nblobs;
      for (uint64_t d = 0; d < dim; ++d) c[d] = static_cast<float>(normal4(centre_seed, blob * dim + d));
      normalize8(c.data(), dim);
      float* o = out + r * dim;
      for (uint64_t d = 0; d < dim; ++d)
        o[d] = c[d] + static_cast<float>(sigma * normal4(noise_seed, i * dim + d));
      normalize8(o, dim);
    }
  });
}

// Integer metadata column uniform in [lo, lo + span): year = 2000 + (u % 30).
void pxf_uniform_int(uint64_t row_begin, uint64_t n, uint64_t seed, int64_t lo, uint64_t span,
                     int64_t* out) {
  for (uint64_t r = 0; r < n; ++r) out[r] = lo + static_cast<int64_t>(stream_at(seed, row_begin + r) % span);
}

}  // extern "C"
