"""Snapshot format and CRC-32C on the CPU.

The oracle's byte-at-a-time CRC (crc.rs:29-79) is pinned by the check values
and properties of crates/proxima-store/src/crc.rs's own tests; the library's
host CRC (slicing-by-8) and its combine are checked against it. The oracle's
codec restatement is checked against the fixed byte layouts the reference's
codec and snapshot tests assert (codec.rs tests, snapshot.rs:120-200), and the
library's host-only snapshot reader (pxc_snapshot_peek) is checked against the
oracle's decode on valid images, on every class of damaged image (including
which error wins when there are two), and on every truncation and single-byte
change of a small image.
"""
import os
import struct

import numpy as np
import pytest

from oracle import pxo
from proxima_b200 import _native as N
from proxima_b200 import snapshot as S
from proxima_b200.errors import Configuration, Corruption


# ---- CRC-32C: crc.rs tests ----

def test_oracle_crc_check_value_and_empty():
    assert pxo.crc32c(b"123456789") == 0xE3069283  # crc.rs:93-99
    assert pxo.crc32c(b"") == 0                     # crc.rs:101-104


def test_oracle_crc_chunking_and_damage():
    data = bytes((i % 256) for i in range(4097))     # crc.rs:106-114
    whole = pxo.crc32c(data)
    for split in (1, 17, 256, 4096):
        assert pxo.crc32c(data[split:], pxo.crc32c(data[:split])) == whole
    clean = pxo.crc32c(bytes([0x5A]) * 512)          # crc.rs:116-126
    for bit in (0, 7, 100, 4095):
        d = bytearray([0x5A]) * 512
        d[bit // 8] ^= 1 << (bit % 8)
        assert pxo.crc32c(d) != clean
    full = bytes(range(200))                         # truncation
    assert pxo.crc32c(full[:-1]) != pxo.crc32c(full)


@pytest.mark.parametrize("n", [0, 1, 3, 7, 8, 9, 15, 16, 17, 255, 256, 257, 4097, 100_003])
def test_library_host_crc_equals_oracle(n):
    rng = np.random.default_rng(n)
    data = rng.integers(0, 256, n + 13, dtype=np.uint8).tobytes()
    for off in (0, 1, 5, 13):  # unaligned starts
        chunk = data[off:off + n]
        assert S.crc32c(chunk) == pxo.crc32c(chunk)
    lib = N.load()
    whole = pxo.crc32c(data)
    for split in (0, 1, n // 2, n, n + 13):
        a, b = pxo.crc32c(data[:split]), pxo.crc32c(data[split:])
        assert lib.pxc_crc32c_combine(a, b, len(data) - split) == whole
        assert S.crc32c(data[split:], a) == whole


# ---- codec layouts ----

def test_metadata_layout_keys_sorted_and_empty_costs_four_bytes():
    # codec.rs tests: metadata_round_trips_and_is_key_ordered, empty_metadata_costs_four_bytes
    assert pxo.encode_metadata_entry({}) == b"\0\0\0\0"
    enc = pxo.encode_metadata_entry({"zeta": 1, "alpha": "x", "mid": True, "f": 2.5})
    keys = []
    pos = 4
    for _ in range(4):
        (kl,) = struct.unpack_from("<I", enc, pos)
        keys.append(enc[pos + 4:pos + 4 + kl].decode())
        pos += 4 + kl
        tag = enc[pos]
        pos += 1 + {1: 4 + 1, 2: 8, 3: 8, 4: 1}[tag]
    assert keys == sorted(keys) == ["alpha", "f", "mid", "zeta"]
    # the product's section encoder writes the same bytes; decode inverts it
    metas = [{}, {"zeta": 1, "alpha": "x", "mid": True, "f": 2.5}, {"neg": -5, "é": "ü"}]
    section = S.encode_metadata(metas, 3)
    assert section == struct.pack("<I", 3) + b"".join(pxo.encode_metadata_entry(m) for m in metas)
    assert S.decode_metadata(section) == metas
    assert S.encode_metadata(None, 2) == struct.pack("<III", 2, 0, 0)


def _parts(n=40, dim=8, m=4, nlist=3, seed=1, trained=True, dead=(3, 7)):
    rng = np.random.default_rng(seed)
    ids = [1000 + i for i in range(n)]
    for d in dead:
        ids[d] = None
    list_of = rng.integers(0, nlist, n).astype(np.uint32)
    for d in dead:
        list_of[d] = 0xFFFFFFFF
    cfg = dict(nlist=nlist, subspaces=m, nprobe=1, rerank=0, seed=0x1FF9C0D, max_iterations=25,
               training_sample=100_000, train_threshold=nlist * 100, retain_vectors=True)
    return dict(dim=dim, metric=pxo.EUCLIDEAN, config=cfg, ids=ids,
                metadata=[{"i": i} if i % 5 == 0 else {} for i in range(n)],
                vectors=rng.standard_normal((n, dim)).astype(np.float32),
                codes=rng.integers(0, 256, (n, m), dtype=np.uint8) if trained else np.zeros(0, np.uint8),
                list_of=list_of if trained else np.zeros(0, np.uint32),
                centroids=rng.standard_normal((nlist, dim)).astype(np.float32) if trained else np.zeros(0, np.float32),
                codebooks=rng.standard_normal(256 * dim).astype(np.float32) if trained else np.zeros(0, np.float32),
                report=dict(sampled=n, coarse_inertia=1.5, coarse_iterations=4, residual_inertia=0.25,
                            populated_lists=nlist, largest_list=20) if trained else None)


def _image(**kw):
    p = _parts(**kw)
    return pxo.snapshot_encode_ivfpq(p["dim"], p["metric"], p["config"], p["ids"], p["metadata"], p["vectors"],
                                     p["codes"], p["list_of"], p["centroids"], p["codebooks"], p["report"]), p


def test_header_layout():
    img, p = _image()
    assert img[:8] == b"PROXSNAP"
    assert struct.unpack_from("<IIIQ", img, 8) == (1, 0x01020304, 0, len(img) - 32)
    assert struct.unpack_from("<I", img, len(img) - 4)[0] == pxo.crc32c(img[28:-4])
    # body: space, kind 3, the 41-byte config, then the id table
    assert struct.unpack_from("<IBB", img, 28) == (8, 1, 3)
    assert struct.unpack_from("<I", img, 28 + 6 + 41)[0] == 40
    dec = pxo.snapshot_decode_ivfpq(img)
    assert dec["ids"] == p["ids"] and dec["metadata"] == p["metadata"]
    assert np.array_equal(dec["codes"], p["codes"].reshape(-1))


# ---- the library's host reader against the oracle ----

@pytest.mark.parametrize("trained", [True, False])
def test_peek_reads_what_the_oracle_wrote(trained):
    img, p = _image(trained=trained)
    info = S.peek(img)
    assert (info.kind, info.dim, info.nslots, info.len) == ("ivfpq", 8, 40, 38)
    assert info.trained == trained and info.has_vectors
    assert info.lists == 3
    assert info.config.nlist == 3 and info.config.subspaces == 4 and info.config.seed == 0x1FF9C0D
    assert (info.report is not None) == trained
    if trained:
        assert info.report["largest_list"] == 20 and info.report["coarse_inertia"] == 1.5
    assert S.decode_metadata(img, info.metadata_offset, info.metadata_bytes) == p["metadata"]


def test_peek_flat_body():
    img = pxo.snapshot_encode_flat(4, pxo.COSINE, [5, None, 9], np.ones((3, 4), np.float32), [{}, {}, {}])
    info = S.peek(img)
    assert (info.kind, info.dim, info.metric, info.nslots, info.len) == ("flat", 4, pxo.COSINE, 3, 2)


def _reseal(img: bytes, body: bytes) -> bytes:
    """A new image around `body` with a correct length and checksum."""
    return img[:20] + struct.pack("<Q", len(body)) + body + struct.pack("<I", pxo.crc32c(body))


def _expect(img, cls, structure=None):
    with pytest.raises(cls) as ei:
        S.peek(img)
    oracle_kind = "corrupt" if cls is Corruption else "config"
    with pytest.raises(pxo.SnapshotError) as eo:
        pxo.snapshot_decode_ivfpq(img)
    assert eo.value.kind == oracle_kind
    if structure is not None:
        got = ei.value.structure if cls is Corruption else ei.value.parameter
        assert got == structure == eo.value.where, (got, eo.value.where)
    return ei.value


def test_header_damage():
    img, _ = _image()
    _expect(img[:31], Corruption, "snapshot header")
    _expect(b"PROXSNAQ" + img[8:], Corruption, "snapshot header")
    _expect(img[:8] + struct.pack("<I", 2) + img[12:], Corruption, "snapshot header")
    _expect(img[:16] + struct.pack("<I", 1) + img[20:], Corruption, "snapshot header")
    _expect(img[:12] + struct.pack("<I", 0x04030201) + img[16:], Corruption, "snapshot header")
    _expect(img + b"\0", Corruption, "snapshot")          # length disagrees
    flipped = bytearray(img)
    flipped[100] ^= 0x10
    e = _expect(bytes(flipped), Corruption, "snapshot")   # checksum
    assert "checksum" in e.detail


def test_body_damage_with_a_valid_checksum():
    img, p = _image()
    body = img[28:-4]
    # bad metric tag, bad kind
    _expect(_reseal(img, body[:4] + b"\x09" + body[5:]), Corruption, "snapshot body")
    _expect(_reseal(img, body[:5] + b"\x07" + body[6:]), Corruption, "snapshot body")
    # an absurd length prefix on the id table
    _expect(_reseal(img, body[:47] + struct.pack("<I", 0xFFFFFFF0) + body[51:]), Corruption, "snapshot body")
    # truncated body, trailing bytes
    _expect(_reseal(img, body[:-3]), Corruption, "snapshot body")
    _expect(_reseal(img, body + b"\0\0"), Corruption, "snapshot body")
    # invalid config: nprobe > nlist (IvfPqConfig::validate)
    cfg_at = 6
    bad = body[:cfg_at + 8] + struct.pack("<I", 99) + body[cfg_at + 12:]
    _expect(_reseal(img, bad), Configuration, "nprobe")


def _variant(**overrides):
    p = _parts()
    p.update(overrides)
    return pxo.snapshot_encode_ivfpq(p["dim"], p["metric"], p["config"], p["ids"], p["metadata"], p["vectors"],
                                     p["codes"], p["list_of"], p["centroids"], p["codebooks"], p["report"])


def test_from_parts_damage():
    p = _parts()
    ids = list(p["ids"])
    ids[9] = ids[2]
    e = _expect(_variant(ids=ids), Corruption, "ivfpq index")
    assert str(ids[2]) in e.detail
    lo = p["list_of"].copy()
    lo[11] = 3
    e = _expect(_variant(list_of=lo), Corruption, "ivfpq index")
    assert "slot 11 names list 3" in e.detail
    lo = p["list_of"].copy()
    lo[3] = 77  # a dead slot's assignment is not checked
    S.peek(_variant(list_of=lo))
    _expect(_variant(metadata=p["metadata"][:-1]), Corruption, "ivfpq index")
    _expect(_variant(vectors=p["vectors"][:-1]), Corruption, "ivfpq index")
    _expect(_variant(codes=p["codes"][:-1]), Corruption, "ivfpq index")
    _expect(_variant(centroids=p["centroids"].reshape(-1)[:-1]), Corruption, "ivfpq centroids")
    _expect(_variant(codebooks=p["codebooks"][:-8]), Corruption, "product quantizer")
    _expect(_variant(metric=pxo.INNER_PRODUCT), Configuration, "metric")


def _outcome_library(img):
    try:
        S.peek(img)
        return ("ok", None)
    except Corruption as e:
        return ("corrupt", e.structure)
    except Configuration as e:
        return ("config", e.parameter)


def _outcome_oracle(img):
    try:
        pxo.snapshot_decode_ivfpq(img)
        return ("ok", None)
    except pxo.SnapshotError as e:
        return (e.kind, e.where)


@pytest.mark.parametrize("trained", [True, False])
def test_every_truncation_and_byte_change_agrees_with_the_oracle(trained):
    """Every truncation of the body and four changes of every body byte (two bit
    flips, 0x00, 0xFF), each resealed with a valid length and checksum so that
    the body parser and from_parts see them: the library's reader accepts
    exactly what the oracle's decode accepts and names the same error class and
    structure or parameter. The index-kind byte is left alone (kinds 1 and 2
    are other bodies)."""
    img, _ = _image(trained=trained)
    body = img[28:-4]
    differ = []
    for cut in range(len(body)):
        x = _reseal(img, body[:cut])
        a, b = _outcome_library(x), _outcome_oracle(x)
        if a != b:
            differ.append(("truncated", cut, a, b))
    for pos in range(len(body)):
        if pos == 5:  # the index kind
            continue
        for v in {body[pos] ^ 0x01, body[pos] ^ 0x80, 0x00, 0xFF} - {body[pos]}:
            x = _reseal(img, body[:pos] + bytes([v]) + body[pos + 1:])
            a, b = _outcome_library(x), _outcome_oracle(x)
            if a != b:
                differ.append(("byte", pos, v, a, b))
    assert not differ, differ[:10]


def test_checksum_wins_over_a_body_error():
    # a body that is both structurally bad and fails its checksum reports the checksum
    img, _ = _image()
    body = bytearray(img[28:-4])
    body[4] = 9  # bad metric tag
    damaged = img[:28] + bytes(body) + img[-4:]
    with pytest.raises(Corruption) as ei:
        S.peek(damaged)
    assert "checksum" in ei.value.detail


def test_write_and_read_snapshot_atomically(tmp_path):
    img, _ = _image()
    path = tmp_path / "index.snap"
    assert S.write_snapshot(path, img) == len(img)
    assert not (tmp_path / "index.tmp").exists()
    assert S.read_snapshot(path) == img
    S.write_snapshot(path, img[:100] + img[100:])  # overwrite in place
    assert S.read_snapshot(path) == img
