// rng.h — host-side ChaCha8Rng as seeded and sampled by the reference's
// k-means++ (crates/proxima-quantize/src/kmeans.rs:150,167,169) and PQ training
// (crates/proxima-quantize/src/product.rs:247), restated from the published
// algorithms of its dependencies (rand_chacha 0.3.1, rand_core 0.6.4,
// rand 0.8.x):
//   * ChaCha with 8 rounds (D. J. Bernstein, "ChaCha, a variant of Salsa20"),
//     64-bit block counter in words 12-13, 64-bit stream id in words 14-15
//     (0 after seeding), four blocks generated per refill into a 64-word
//     buffer; the position in the key stream counts u32 words (get_word_pos);
//   * seed_from_u64: PCG32 (XSH-RR, M. O'Neill 2014) expanding the u64 into
//     the 32-byte key, one u32 per step;
//   * next_u64 = two consecutive u32 words, low word first (a refill may fall
//     between them);
//   * gen_range(0..n) for usize: widening multiply with rejection zone;
//   * gen_range(lo..hi) for f64: 52 random mantissa bits in [1,2), minus 1,
//     times the span, plus lo, redrawn if it reaches hi.
// The block function is pinned by published known answers (RFC 8439's
// 20-round block and key-stream vectors, the 8-round zero-key key stream) and
// the PCG32 output function by the PCG reference generator's demo output.
// No draw of the Rust crates themselves is pinned (there is no Rust toolchain
// to produce one), so the seed expansion and range sampling rest on the
// published algorithms only.
#pragma once
#include <stdint.h>

#include <cmath>
#include <cstring>

namespace pxc {

// One ChaCha block: 16 words of key stream for (key, 64-bit block counter,
// 64-bit stream id) after `rounds` rounds (even). Words 12-13 hold the
// counter and 14-15 the stream, as in Bernstein's original layout; RFC 8439's
// 32-bit counter + 96-bit nonce is the same state with counter = nonce[0] << 32 | count.
inline void chacha_block(const uint32_t key[8], uint64_t counter, uint64_t stream, int rounds, uint32_t out[16]) {
  const uint32_t s[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u, key[0], key[1], key[2], key[3],
                          key[4],      key[5],      key[6],      key[7],      static_cast<uint32_t>(counter),
                          static_cast<uint32_t>(counter >> 32), static_cast<uint32_t>(stream),
                          static_cast<uint32_t>(stream >> 32)};
  uint32_t x[16];
  std::memcpy(x, s, sizeof(x));
  auto rotl = [](uint32_t v, int r) { return (v << r) | (v >> (32 - r)); };
  auto quarter = [&](int a, int b, int c, int d) {
    x[a] += x[b];
    x[d] = rotl(x[d] ^ x[a], 16);
    x[c] += x[d];
    x[b] = rotl(x[b] ^ x[c], 12);
    x[a] += x[b];
    x[d] = rotl(x[d] ^ x[a], 8);
    x[c] += x[d];
    x[b] = rotl(x[b] ^ x[c], 7);
  };
  for (int round = 0; round < rounds; round += 2) {
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

// PCG32 step and XSH-RR output as rand_core's seed_from_u64 uses them: the
// state advances first (multiplier 6364136223846793005, increment
// 11634580027462260723) and the output is taken from the new state.
inline uint32_t pcg32_xsh_rr(uint64_t state) {
  const uint32_t xs = static_cast<uint32_t>(((state >> 18) ^ state) >> 27);
  const uint32_t rot = static_cast<uint32_t>(state >> 59);
  return (xs >> rot) | (xs << ((32 - rot) & 31));
}

class ChaCha8 {
 public:
  // ChaCha8Rng::seed_from_u64: eight PCG32 outputs, little-endian, form the key.
  explicit ChaCha8(uint64_t seed) {
    const uint64_t mul = 6364136223846793005ull, inc = 11634580027462260723ull;
    uint64_t state = seed;
    for (int i = 0; i < 8; ++i) {
      state = state * mul + inc;
      key_[i] = pcg32_xsh_rr(state);
    }
  }

  // ChaCha8Rng::from_seed(seed) + set_stream(stream) + set_word_pos(word_pos),
  // word_pos = word_pos_hi * 2^64 + word_pos_lo (a 68-bit position).
  ChaCha8(const uint8_t seed[32], uint64_t stream, uint64_t word_pos_lo, uint64_t word_pos_hi) {
    for (int i = 0; i < 8; ++i)
      key_[i] = static_cast<uint32_t>(seed[4 * i]) | static_cast<uint32_t>(seed[4 * i + 1]) << 8 |
                static_cast<uint32_t>(seed[4 * i + 2]) << 16 | static_cast<uint32_t>(seed[4 * i + 3]) << 24;
    stream_ = stream;
    const uint64_t block = (word_pos_hi << 60) | (word_pos_lo >> 4);
    counter_ = block;
    refill();
    index_ = static_cast<uint32_t>(word_pos_lo & 15);
  }

  // The inverse of the constructor above: get_seed, get_stream, get_word_pos.
  void state(uint8_t seed[32], uint64_t* stream, uint64_t* word_pos_lo, uint64_t* word_pos_hi) const {
    for (int i = 0; i < 8; ++i)
      for (int b = 0; b < 4; ++b) seed[4 * i + b] = static_cast<uint8_t>(key_[i] >> (8 * b));
    *stream = stream_;
    // the buffer holds blocks [counter_ - 4, counter_); rand_chacha wraps the
    // block number in 64 bits before scaling it to words
    const uint64_t block = (counter_ - 4) + index_ / 16;
    *word_pos_lo = (block << 4) | (index_ % 16);
    *word_pos_hi = block >> 60;
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
  void refill() {
    for (int b = 0; b < 4; ++b) chacha_block(key_, counter_ + b, stream_, 8, buf_ + 16 * b);
    counter_ += 4;
    index_ = 0;
  }

  uint32_t key_[8];
  uint64_t stream_ = 0;
  uint64_t counter_ = 0;  // next block to generate
  uint32_t buf_[64] = {0};
  uint32_t index_ = 64;  // next word of buf_ (64: empty)
};

}  // namespace pxc
