"""IVF-PQ snapshots straight to and from the device (pxc_ivfpq_snapshot_save /
_load) and CRC-32C on the device (pxc_crc32c_device), against the oracle's
restatement of the codec and of crc.rs.

* The device CRC equals the oracle's byte-at-a-time CRC at every length
  around the kernel's run, step and alignment boundaries.
* A saved image is byte-for-byte the oracle's encoding of the same parts
  (snapshot.rs:120-200), and re-saving a loaded index reproduces it.
* A loaded index answers every query as the saved one did, ids and f32 bits,
  and as the oracle's search over the oracle's decode of the image.
* Damaged images fail with the class and structure the host reader and the
  oracle name, the checksum first.
"""
import numpy as np
import pytest
import torch

from oracle import pxo
from proxima_b200 import fixtures
from proxima_b200 import snapshot as S
from proxima_b200.errors import Configuration, Corruption
from proxima_b200.filters import MetadataFilter
from proxima_b200.ivfpq import IvfPqIndex

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [0, 1, 3, 15, 16, 17, 255, 256, 257, 511, 512, 513, 4095, 131071, 131072, 131073,
                               262143, 262144, 262145, (1 << 20) + 5, (3 << 20) + 77])
def test_device_crc_equals_the_oracle(n):
    rng = np.random.default_rng(n)
    host = rng.integers(0, 256, n + 16, dtype=np.uint8)
    dev = torch.from_numpy(host).cuda()
    for off in (0, 1, 7, 15):
        want = pxo.crc32c(host[off:off + n].tobytes())
        assert S.crc32c_device(dev[off:off + n]) == want, (n, off)


def test_device_crc_large():
    n = (96 << 20) + 12345  # several blocks of several steps each
    host = np.random.default_rng(5).integers(0, 256, n, dtype=np.uint8)
    assert S.crc32c_device(torch.from_numpy(host).cuda()) == S.crc32c(host)
    assert S.crc32c(host[:1 << 20]) == pxo.crc32c(host[:1 << 20].tobytes())


def _trained(n=6000, dim=32, nlist=32, m=8, dead=range(0, 6000, 11)):
    data = fixtures.blobs_f32(n, dim, 32, 3, 4)
    ids = np.arange(n, dtype=np.uint64) * 3 + 7
    live = np.ones(n, np.uint8)
    live[list(dead)] = 0
    idx = IvfPqIndex(dim, nlist, m)
    idx.set_store(data, ids=ids, live=live)
    idx.train(training_sample=3000, max_iterations=8, seed=5)
    metas = [{"g": int(i % 4), "name": f"v{i}"} if live[i] else {} for i in range(n)]
    idx.set_metadata(metas)
    return idx, data, ids, live, metas


def _oracle_image(idx, data, ids, live, metas, cfg, with_vectors=True, report=True):
    cent, books, list_of, codes = idx.parts()
    rep = {f: idx.report[f] for f in ("sampled", "coarse_inertia", "coarse_iterations", "residual_inertia",
                                      "populated_lists", "largest_list")} if report else None
    return pxo.snapshot_encode_ivfpq(
        idx.dim, pxo.EUCLIDEAN, vars(cfg), [int(i) if l else None for i, l in zip(ids, live)], metas,
        data if with_vectors else np.zeros(0, np.float32), codes, list_of, cent, books, rep)


def test_save_is_the_oracle_encoding_and_load_round_trips():
    idx, data, ids, live, metas = _trained()
    cfg = S.IvfPqConfig(idx.nlist, idx.m, nprobe=4)
    img = S.save_ivfpq(idx, cfg)
    assert img == _oracle_image(idx, data, ids, live, metas, cfg)
    idx2, info = S.load_ivfpq(img)
    assert (info.kind, info.nslots, info.len, info.lists, info.trained) == ("ivfpq", 6000, int(live.sum()), 32, True)
    assert S.save_ivfpq(idx2) == img  # config, report and metadata come back with the index
    for part_a, part_b in zip(idx.parts(), idx2.parts()):
        assert np.array_equal(part_a, part_b)
    idx2.close()
    idx.close()


@pytest.mark.parametrize("nprobe,rerank", [(4, 0), (8, 60), (32, 200)])
def test_loaded_index_answers_as_the_saved_one(nprobe, rerank):
    idx, data, ids, live, metas = _trained()
    img = S.save_ivfpq(idx, S.IvfPqConfig(idx.nlist, idx.m))
    idx2, _ = S.load_ivfpq(img)
    q = fixtures.blobs_f32(300, 32, 32, 3, 9)
    a = idx.search_batch(q, 10, nprobe, rerank)
    b = idx2.search_batch(q, 10, nprobe, rerank)
    assert np.array_equal(a[2], b[2])
    for q_i in range(len(q)):
        n_i = a[2][q_i]
        assert np.array_equal(a[0][q_i, :n_i], b[0][q_i, :n_i])
        assert np.array_equal(a[1][q_i, :n_i].view(np.uint32), b[1][q_i, :n_i].view(np.uint32))
    # and as the oracle searches the oracle's decode of the image
    dec = pxo.snapshot_decode_ivfpq(img)
    lv = np.array([i is not None for i in dec["ids"]], np.uint8)
    idv = np.array([i or 0 for i in dec["ids"]], np.uint64)
    ri, rd, rl = pxo.ivfpq_search(dec["vectors"].reshape(-1, 32), dec["centroids"].reshape(-1, 32),
                                  dec["codebooks"], 8, dec["list_of"], dec["codes"].reshape(-1, 8), q, 10, nprobe,
                                  rerank, ids=idv, live=lv)
    assert np.array_equal(rl, b[2])
    for q_i in range(len(q)):
        assert np.array_equal(ri[q_i, :rl[q_i]], b[0][q_i, :rl[q_i]])
        assert np.array_equal(rd[q_i, :rl[q_i]].view(np.uint32), b[1][q_i, :rl[q_i]].view(np.uint32))
    idx.close()
    idx2.close()


def test_metadata_filters_survive_the_round_trip():
    idx, data, ids, live, metas = _trained()
    idx2, _ = S.load_ivfpq(S.save_ivfpq(idx, S.IvfPqConfig(idx.nlist, idx.m)))
    q = fixtures.blobs_f32(64, 32, 32, 3, 10)
    flt = MetadataFilter.parse({"g": {"in": [1, 3]}})
    a = idx.search_where(q, 10, 8, 50, flt)
    b = idx2.search_where(q, 10, 8, 50, flt)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
    idx.close()
    idx2.close()


def test_untrained_and_codes_only_indexes():
    data = fixtures.blobs_f32(500, 16, 8, 3, 4)
    # untrained: vectors only
    u = IvfPqIndex(16, 8, 4)
    u.set_store(data)
    cfg = S.IvfPqConfig(8, 4)
    img = S.save_ivfpq(u, cfg)
    dec = pxo.snapshot_decode_ivfpq(img)
    assert dec["centroids"].size == 0 and dec["codes"].size == 0 and dec["report"] is None
    assert np.array_equal(dec["vectors"].reshape(-1, 16), data)
    u2, info = S.load_ivfpq(img)
    assert not info.trained and info.lists == 8 and info.has_vectors
    assert S.save_ivfpq(u2) == img
    # retain_vectors off: parts and codes, no vectors
    cent, books, list_of, codes, _ = pxo.ivfpq_train(data, 8, 4, 4, 500, 0x77)
    r = IvfPqIndex(16, len(cent), 4)
    r.from_parts(cent, books)
    r.set_store(None, ids=np.arange(500, dtype=np.uint64), nslots=500)
    r.set_codes(list_of, codes)
    cfg = S.IvfPqConfig(8, 4, retain_vectors=False)
    img = S.save_ivfpq(r, cfg)
    dec = pxo.snapshot_decode_ivfpq(img)
    assert dec["vectors"].size == 0 and np.array_equal(dec["codes"].reshape(-1, 4), codes)
    r2, info = S.load_ivfpq(img)
    assert not info.has_vectors and info.config.retain_vectors is False
    q = fixtures.blobs_f32(50, 16, 8, 3, 6)
    a, b = r.search_batch(q, 5, 4), r2.search_batch(q, 5, 4)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
    for h in (u, u2, r, r2):
        h.close()


def _load_error(img):
    with pytest.raises((Corruption, Configuration)) as ei:
        S.load_ivfpq(img)
    with pytest.raises(type(ei.value)) as ep:
        S.peek(img)
    return ei.value, ep.value


def test_damaged_images_fail_as_the_host_reader_says():
    idx, data, ids, live, metas = _trained(n=2000, dead=range(0, 2000, 9))
    cfg = S.IvfPqConfig(idx.nlist, idx.m)
    good = _oracle_image(idx, data, ids, live, metas, cfg)
    assert S.save_ivfpq(idx, cfg) == good
    cent, books, list_of, codes = idx.parts()
    live_ids = [int(i) if l else None for i, l in zip(ids, live)]
    enc = lambda **kw: pxo.snapshot_encode_ivfpq(
        32, pxo.EUCLIDEAN, vars(cfg), kw.get("ids", live_ids), metas, data, codes, kw.get("list_of", list_of),
        cent, books, None)
    dup = list(live_ids)
    dup[1500] = dup[20]
    e, p = _load_error(enc(ids=dup))
    assert isinstance(e, Corruption) and e.structure == p.structure == "ivfpq index" and str(dup[20]) in e.detail
    lo = list_of.copy()
    lo[1001] = 999
    e, p = _load_error(enc(list_of=lo))
    assert e.structure == "ivfpq index" and "slot 1001 names list 999" in e.detail
    # a flipped bit inside the vectors: only the device CRC sees it
    body_flip = bytearray(good)
    body_flip[len(good) // 3] ^= 0x04
    e, p = _load_error(bytes(body_flip))
    assert "checksum" in e.detail and "checksum" in p.detail
    # both a duplicate id and a bad checksum: the checksum wins
    both = bytearray(enc(ids=dup))
    both[len(both) // 3] ^= 0x04
    e, _ = _load_error(bytes(both))
    assert "checksum" in e.detail
    # another kind of index
    flat = pxo.snapshot_encode_flat(4, pxo.EUCLIDEAN, [1, 2], np.ones((2, 4), np.float32), [{}, {}])
    with pytest.raises(Configuration):
        S.load_ivfpq(flat)
    idx.close()


def test_large_arrays_take_the_staged_copies():
    """Vectors of 12 MB move through the pinned ring in both directions (8 MiB
    chunks, a partial last one): the image still equals the oracle's encoding
    and the reload equals the saved index."""
    n, dim, m = 48_000, 64, 16
    data = fixtures.blobs_f32(n, dim, 64, 5, 6)
    idx = IvfPqIndex(dim, 64, m)
    idx.set_store(data)
    idx.train(training_sample=8000, max_iterations=5, seed=9)
    cfg = S.IvfPqConfig(idx.nlist, m)
    img = S.save_ivfpq(idx, cfg)
    cent, books, list_of, codes = idx.parts()
    rep = {f: idx.report[f] for f in ("sampled", "coarse_inertia", "coarse_iterations", "residual_inertia",
                                      "populated_lists", "largest_list")}
    want = pxo.snapshot_encode_ivfpq(dim, pxo.EUCLIDEAN, vars(cfg), list(range(n)), [{}] * n, data, codes, list_of,
                                     cent, books, rep)
    assert img == want
    idx2, _ = S.load_ivfpq(bytes(img))
    for a, b in zip(idx.parts(), idx2.parts()):
        assert np.array_equal(a, b)
    q = fixtures.blobs_f32(100, dim, 64, 5, 7)
    for x, y in zip(idx.search_batch(q, 10, 8, 100), idx2.search_batch(q, 10, 8, 100)):
        assert np.array_equal(x, y)
    idx.close()
    idx2.close()
