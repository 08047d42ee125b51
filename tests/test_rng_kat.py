"""Known answers for the generator the reference's training draws from.

k-means++ seeding (crates/proxima-quantize/src/kmeans.rs:146-194), PQ training
(product.rs:247) and IVF training (crates/proxima-index/src/ivfpq.rs:770) draw
from rand_chacha 0.3.1's ChaCha8Rng, seeded by rand_core 0.6.4's
seed_from_u64. The reference pins no draw, so the pins here are published
known answers for the building blocks, checked in both the native library
(the product, host-side code) and the oracle:

* the ChaCha block function, against RFC 8439 (section 2.3.2's block with
  its nonce, appendix A.1's key-stream vectors) at 20 rounds, and against the
  published 8-round key stream for the all-zero key and IV;
* ChaCha20 over a seed laid out as rand_chacha lays it out (little-endian
  key words), against the first word rand_chacha's own documentation gives;
* PCG32's XSH-RR output function and multiplier, against the PCG reference
  generator's demo output (pcg32_srandom_r(42, 54)); seed_from_u64 then
  reuses that function with rand_core's published increment;
* the generator's word position (get_word_pos / set_word_pos) round trip.

These run on the host: no GPU is needed.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import pxo
from proxima_b200 import _native as N
from proxima_b200.quantize import ChaCha8Rng, chacha_block

MASK64 = (1 << 64) - 1


def _words_le(hexstr: str) -> list[int]:
    b = bytes.fromhex(hexstr)
    return [int.from_bytes(b[i:i + 4], "little") for i in range(0, len(b), 4)]


def _oracle_block(key, counter, stream, rounds):
    k = np.ascontiguousarray(key, np.uint32)
    out = np.zeros(16, np.uint32)
    pxo.lib().pxo_chacha_block(k.ctypes.data, counter, stream, rounds, out.ctypes.data)
    return out


def _both(key, counter, stream, rounds):
    a = chacha_block(key, counter, stream, rounds)
    b = _oracle_block(key, counter, stream, rounds)
    assert np.array_equal(a, b), "library and oracle block functions differ"
    return [int(x) for x in a]


# RFC 8439 2.3.2: key 00 01 .. 1f, nonce 00:00:00:09:00:00:00:4a:00:00:00:00,
# block count 1. State words 12-15 = 1, 0x09000000, 0x4a000000, 0: in the
# 64-bit counter / 64-bit stream layout, counter = 0x09000000 << 32 | 1 and
# stream = 0x4a000000.
RFC8439_232 = [
    0xE4E7F110, 0x15593BD1, 0x1FDD0F50, 0xC47120A3,
    0xC7F4D1C7, 0x0368C033, 0x9AAA2204, 0x4E6CD4C3,
    0x466482D2, 0x09AA9F07, 0x05D7C214, 0xA2028BD9,
    0xD19C12B5, 0xB94E16DE, 0xE883D0CB, 0x4E3C50A2,
]
# RFC 8439 A.1 test vector #1: all-zero key and nonce, block count 0.
RFC8439_A1_1 = _words_le(
    "76b8e0ada0f13d90405d6ae55386bd28bdd219b8a08ded1aa836efcc8b770dc7"
    "da41597c5157488d7724e03fb8d84a376a43b8f41518a11cc387b669b2ee6586")
# 8 rounds, all-zero 256-bit key and IV: the first 64 key-stream bytes.
CHACHA8_ZERO = _words_le(
    "3e00ef2f895f40d67f5bb8e81f09a5a12c840ec3ce9a7f3b181be188ef711a1e"
    "984ce172b9216f419f445367456d5619314a42a3da86b001387bfdb80e0cfe42")


def test_chacha20_rfc8439_block():
    key = [int.from_bytes(bytes(range(4 * i, 4 * i + 4)), "little") for i in range(8)]
    assert _both(key, (0x09000000 << 32) | 1, 0x4A000000, 20) == RFC8439_232


def test_chacha20_rfc8439_zero_key_stream():
    assert _both([0] * 8, 0, 0, 20) == RFC8439_A1_1


def test_chacha8_zero_key_stream():
    assert _both([0] * 8, 0, 0, 8) == CHACHA8_ZERO


def test_rand_chacha_seed_layout():
    """rand_chacha documents ChaChaRng::from_seed([0,0,0,0, 0,0,0,0, 1,0,0,0, 0,0,0,0,
    2,0,0,0, 0,0,0,0, 3,0,0,0, 0,0,0,0]).next_u32() == 137206642 (20 rounds): the seed
    bytes become key words little-endian, the first word comes from block 0."""
    seed = bytes([0] * 8 + [1] + [0] * 7 + [2] + [0] * 7 + [3] + [0] * 7)
    key = [int.from_bytes(seed[4 * i:4 * i + 4], "little") for i in range(8)]
    assert _both(key, 0, 0, 20)[0] == 137206642


def _xsh_rr(state: int) -> int:
    xs = (((state >> 18) ^ state) >> 27) & 0xFFFFFFFF
    rot = state >> 59
    return ((xs >> rot) | (xs << ((32 - rot) & 31))) & 0xFFFFFFFF


PCG_MUL = 6364136223846793005


def test_pcg32_output_function_matches_reference_demo():
    """pcg32_srandom_r(42, 54) then six pcg32_random_r calls (PCG's demo program)."""
    inc = (54 << 1) | 1
    state = 0
    state = (state * PCG_MUL + inc) & MASK64
    state = (state + 42) & MASK64
    state = (state * PCG_MUL + inc) & MASK64
    out = []
    for _ in range(6):
        old = state
        state = (old * PCG_MUL + inc) & MASK64
        out.append(_xsh_rr(old))
    assert out == [0xA15C02B7, 0x7B47F409, 0xBA1D3330, 0x83D2F293, 0xBFA4784B, 0xCBED606E]


@pytest.mark.parametrize("seed", [0, 1, 42, 0x1FF9C0D, 0x5EED, MASK64])
def test_seed_from_u64_is_pcg32_with_rand_core_increment(seed):
    """rand_core 0.6.4 seed_from_u64: advance (x MUL + 11634580027462260723), output
    XSH-RR of the new state, eight words little-endian into the 32-byte seed."""
    inc = 11634580027462260723
    st = seed
    want = b""
    for _ in range(8):
        st = (st * PCG_MUL + inc) & MASK64
        want += _xsh_rr(st).to_bytes(4, "little")
    rng = ChaCha8Rng.seed_from_u64(seed)
    assert rng.get_seed() == want and rng.get_stream() == 0 and rng.get_word_pos() == 0
    # the oracle's generator holds the same key
    r = pxo.Rng()
    pxo.lib().pxo_rng_seed_from_u64(C.byref(r), seed)
    assert bytes(np.array(list(r.key), np.uint32).astype("<u4").tobytes()) == want


def test_stream_and_word_position():
    """next_u32 walks the 8-round key stream block by block; get_word_pos counts
    words; a generator rebuilt at a word position continues the same stream."""
    rng = ChaCha8Rng.seed_from_u64(7)
    key = np.frombuffer(rng.get_seed(), "<u4")
    want = np.concatenate([chacha_block(key, b, 0, 8) for b in range(10)])
    got = rng.next_u32_array(37)
    assert np.array_equal(got, want[:37]) and rng.get_word_pos() == 37
    rest = ChaCha8Rng.from_seed(rng.get_seed(), 0, 37).next_u32_array(100)
    assert np.array_equal(rest, want[37:137])
    assert np.array_equal(rng.next_u32_array(100), want[37:137]) and rng.get_word_pos() == 137
    # a non-zero stream id feeds words 14-15
    s = ChaCha8Rng.from_seed(rng.get_seed(), 5, 0)
    assert np.array_equal(s.next_u32_array(16), chacha_block(key, 0, 5, 8))
    # the oracle's generator draws the same words
    r = pxo.Rng()
    pxo.lib().pxo_rng_seed_from_u64(C.byref(r), 7)
    assert [pxo.lib().pxo_rng_next_u32(C.byref(r)) for _ in range(137)] == [int(x) for x in want[:137]]


def test_range_draws_match_oracle():
    """gen_range(0..n) for usize and gen_range(lo..hi) for f64 (rand 0.8) in the
    library equal the oracle's draw for draw (both restate rand's documented
    algorithms; k-means++ makes exactly these calls)."""
    rng = ChaCha8Rng.seed_from_u64(0xC3)
    r = pxo.Rng()
    pxo.lib().pxo_rng_seed_from_u64(C.byref(r), 0xC3)
    for bound in (1, 2, 3, 1000, 1_000_000, (1 << 63) + 5):
        assert rng.gen_index(bound) == pxo.lib().pxo_rng_gen_range_usize(C.byref(r), bound)
    for lo, hi in ((0.0, 1.0), (0.0, 1e-300), (-3.5, 7.25), (0.0, 123456.789)):
        assert rng.gen_f64(lo, hi) == pxo.lib().pxo_rng_gen_range_f64(C.byref(r), lo, hi)


def test_rng_argument_errors():
    from proxima_b200.errors import Configuration

    with pytest.raises(Configuration):
        ChaCha8Rng.seed_from_u64(1).gen_index(0)
    with pytest.raises(Configuration):
        ChaCha8Rng.seed_from_u64(1).gen_f64(1.0, 1.0)
    bad = N.PxcRng()
    bad.word_pos_hi = 16
    with pytest.raises(Configuration):
        ChaCha8Rng(bad).next_u32()
