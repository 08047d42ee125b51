// rng.h — host-side ChaCha8Rng as seeded and sampled by the reference's
// k-means++ (crates/proxima-quantize/src/kmeans.rs:150,167,169) and PQ training
// (crates/proxima-quantize/src/product.rs:247), restated from the published
// algorithms of its dependencies (rand_chacha 0.3.1, rand_core 0.6.4,
// rand 0.8.x):
//   * ChaCha with 8 rounds (D. J. Bernstein, "ChaCha, a variant of Salsa20"),
//     64-bit block counter in words 12-13, stream id 0 in words 14-15, four
//     blocks generated per refill into a 64-word buffer;
//   * seed_from_u64: PCG32 (XSH-RR, M. O'Neill 2014) expanding the u64 into
//     the 32-byte key, one u32 per step;
//   * next_u64 = two consecutive u32 words, low word first (a refill may fall
//     between them);
//   * gen_range(0..n) for usize: widening multiply with rejection zone;
//   * gen_range(lo..hi) for f64: 52 random mantissa bits in [1,2), minus 1,
//     times the span, plus lo, redrawn if it reaches hi.
// No draw of the real crates is pinned here (there is no Rust toolchain to
// produce one), so agreement with them is unpinned.
#pragma once
#include <stdint.h>

#include <cmath>
#include <cstring>

namespace pxc {

class ChaCha8 {
 public:
  explicit ChaCha8(uint64_t seed) {
    const uint64_t mul = 6364136223846793005ull, inc = 11634580027462260723ull;
    uint64_t state = seed;
    for (int i = 0; i < 8; ++i) {
      state = state * mul + inc;
      uint32_t xs = static_cast<uint32_t>(((state >> 18) ^ state) >> 27);
      uint32_t rot = static_cast<uint32_t>(state >> 59);
      key_[i] = (xs >> rot) | (xs << ((32 - rot) & 31));
    }
  }

  uint32_t next_u32() {
    if (index_ >= 64) refill();
    return buf_[index_++];
  }

  uint64_t next_u64() {
    uint64_t lo = next_u32();
    uint64_t hi = next_u32();
    return (hi << 32) | lo;
  }

  // Uniform in [0, n), n >= 1.
  uint64_t gen_index(uint64_t n) {
    if (n == 0) return next_u64();
    const uint64_t zone = (n << __builtin_clzll(n)) - 1;
    for (;;) {
      const uint64_t v = next_u64();
      const unsigned __int128 m = static_cast<unsigned __int128>(v) * n;
      if (static_cast<uint64_t>(m) <= zone) return static_cast<uint64_t>(m >> 64);
    }
  }

  // Uniform in [lo, hi), hi > lo.
  double gen_f64(double lo, double hi) {
    double span = hi - lo;
    for (;;) {
      const uint64_t bits = (next_u64() >> 12) | 0x3FF0000000000000ull;
      double v12;
      std::memcpy(&v12, &bits, 8);
      const double r = (v12 - 1.0) * span + lo;
      if (r < hi) return r;
      span = std::nextafter(span, 0.0);
    }
  }

 private:
  static uint32_t rotl(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

  void block(uint64_t counter, uint32_t* out) const {
    uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, key_[0], key_[1], key_[2], key_[3],
                      key_[4],     key_[5],     key_[6],     key_[7],     static_cast<uint32_t>(counter),
                      static_cast<uint32_t>(counter >> 32), 0u, 0u};
    uint32_t x[16];
    std::memcpy(x, s, sizeof(x));
    auto quarter = [&x](int a, int b, int c, int d) {
      x[a] += x[b];
      x[d] = rotl(x[d] ^ x[a], 16);
      x[c] += x[d];
      x[b] = rotl(x[b] ^ x[c], 12);
      x[a] += x[b];
      x[d] = rotl(x[d] ^ x[a], 8);
      x[c] += x[d];
      x[b] = rotl(x[b] ^ x[c], 7);
    };
    for (int round = 0; round < 8; round += 2) {
      quarter(0, 4, 8, 12);
      quarter(1, 5, 9, 13);
      quarter(2, 6, 10, 14);
      quarter(3, 7, 11, 15);
      quarter(0, 5, 10, 15);
      quarter(1, 6, 11, 12);
      quarter(2, 7, 8, 13);
      quarter(3, 4, 9, 14);
    }
    for (int i = 0; i < 16; ++i) out[i] = x[i] + s[i];
  }

  void refill() {
    for (int b = 0; b < 4; ++b) block(counter_ + b, buf_ + 16 * b);
    counter_ += 4;
    index_ = 0;
  }

  uint32_t key_[8];
  uint64_t counter_ = 0;
  uint32_t buf_[64] = {0};
  uint32_t index_ = 64;
};

}  // namespace pxc
