"""Persisted repacked-expert cache (storage.llm_b200/expert_cache.py) on the
CPU: the file format round trip, its checks, and the residency choice
between a cached record and the repacking upload (against a fake engine)."""
import os

import numpy as np
import pytest


@pytest.fixture(scope="module")
def ec(pkg):
    import moe_b200.expert_cache as m
    return m


def _records(ec, rng, hidden, inter, n):
    rb = ec.record_bytes(hidden, inter)
    return [(li, e, int(rng.integers(0, 2**63)), rng.integers(0, 256, rb, dtype=np.uint8))
            for li, e in n]


def test_record_bytes_matches_the_library(ec, pkg):
    import moe_b200.lib as L
    lib = L.load()
    for h, i in ((64, 96), (1024, 512), (2880, 2880), (7168, 2048), (896, 384), (100, 30)):
        assert ec.record_bytes(h, i) == lib.moe_b200_expert_record_bytes(h, i) > 0
    assert ec.record_bytes(0, 64) == lib.moe_b200_expert_record_bytes(0, 64) == 0


def test_round_trip(ec, tmp_path):
    rng = np.random.default_rng(0)
    recs = _records(ec, rng, 256, 384, [(0, 0), (0, 3), (0, -1), (2, 1)])
    path = str(tmp_path / "m.b200cache")
    assert ec.write_cache(path, 256, 384, recs) == 4
    f = ec.CacheFile(path)
    assert (f.hidden, f.intermediate, f.record_bytes) == (256, 384, ec.record_bytes(256, 384))
    for layer, expert, key, rec in recs:
        assert f.entries[(layer, expert)].offset % ec.ALIGN == 0
        got = f.get(layer, expert, key)
        assert got is not None and np.array_equal(got, rec)
        assert np.array_equal(f.get(layer, expert), rec)      # no key: any record
        assert f.get(layer, expert, key ^ 1) is None          # other source bytes
    assert f.get(0, 1) is None and f.get(1, 0) is None
    f.close()
    assert os.path.getsize(path) % ec.ALIGN == 0


def test_empty_cache(ec, tmp_path):
    path = str(tmp_path / "e.b200cache")
    assert ec.write_cache(path, 128, 128, []) == 0
    f = ec.CacheFile(path)
    assert f.entries == {} and f.get(0, 0) is None


def test_write_checks(ec, tmp_path):
    rng = np.random.default_rng(1)
    rb = ec.record_bytes(128, 256)
    path = str(tmp_path / "w.b200cache")
    with pytest.raises(ec.CacheError):
        ec.write_cache(path, 128, 256, [(0, 0, 1, np.zeros(rb - 1, np.uint8))])
    with pytest.raises(ec.CacheError):
        rec = rng.integers(0, 256, rb, dtype=np.uint8)
        ec.write_cache(path, 128, 256, [(0, 0, 1, rec), (0, 0, 2, rec)])
    with pytest.raises(ec.CacheError):
        ec.write_cache(path, 0, 256, [])
    assert not os.path.exists(path)


def _corrupt(path, offset, n=1):
    with open(path, "r+b") as fh:
        fh.seek(offset)
        b = bytearray(fh.read(n))
        fh.seek(offset)
        fh.write(bytes(x ^ 0xFF for x in b))


def test_read_checks(ec, tmp_path):
    rng = np.random.default_rng(2)
    recs = _records(ec, rng, 128, 128, [(0, 0), (0, 1)])
    path = str(tmp_path / "r.b200cache")
    ec.write_cache(path, 128, 128, recs)
    # a flipped record byte fails that record's checksum, not the other's
    off = ec.CacheFile(path).entries[(0, 1)].offset
    _corrupt(path, off + 17)
    f = ec.CacheFile(path)
    assert np.array_equal(f.get(0, 0, recs[0][2]), recs[0][3])
    with pytest.raises(ec.CacheError, match="checksum"):
        f.get(0, 1, recs[1][2])
    with pytest.raises(ec.CacheError, match="checksum"):
        f.verify_all()
    assert f.get(0, 1, recs[1][2], verify=False) is not None   # unchecked reads are the caller's choice
    # a damaged entry table, a wrong magic and a truncated file are refused
    ec.write_cache(path, 128, 128, recs)
    _corrupt(path, ec.HEADER_BYTES + 3)
    with pytest.raises(ec.CacheError, match="entry table"):
        ec.CacheFile(path)
    ec.write_cache(path, 128, 128, recs)
    _corrupt(path, 0)
    with pytest.raises(ec.CacheError, match="not a repacked-expert cache"):
        ec.CacheFile(path)
    ec.write_cache(path, 128, 128, recs)
    size = os.path.getsize(path)
    with open(path, "r+b") as fh:
        fh.truncate(size - ec.ALIGN)
    with pytest.raises(ec.CacheError, match="outside the file"):
        ec.CacheFile(path)
    with open(path, "r+b") as fh:
        fh.truncate(100)
    with pytest.raises(ec.CacheError, match="shorter than the header"):
        ec.CacheFile(path)


def test_source_key(ec):
    rng = np.random.default_rng(3)
    g, u, d = (rng.integers(0, 256, 170, dtype=np.uint8) for _ in range(3))
    k = ec.source_key(g, u, d)
    assert k == ec.source_key(g.copy(), u.copy(), d.copy())
    g2 = g.copy()
    g2[5] ^= 1
    assert ec.source_key(g2, u, d) != k
    assert ec.source_key(u, g, d) != k
    # the same concatenated bytes split differently are another expert
    assert ec.source_key(g[:-1], np.concatenate([g[-1:], u]), d) != k


class FakeEngine:
    def __init__(self):
        self.calls = []

    def import_expert(self, layer, expert, rec, hidden, intermediate, on_device=False):
        self.calls.append(("import", layer, expert, bytes(rec[:4])))

    def upload_expert(self, layer, expert, gate, up, down, hidden, intermediate, on_device=False):
        self.calls.append(("upload", layer, expert))

    def export_expert(self, layer, expert, hidden, intermediate):
        rb = self.rb
        return np.full(rb, (layer * 16 + expert) & 0xFF, np.uint8)


def test_make_resident_prefers_a_matching_record(ec, tmp_path):
    rng = np.random.default_rng(4)
    H, I = 128, 256
    src = {e: tuple(rng.integers(0, 256, 64, dtype=np.uint8) for _ in range(3)) for e in (0, 1, -1)}
    eng = FakeEngine()
    eng.rb = ec.record_bytes(H, I)
    path = str(tmp_path / "res.b200cache")
    keys = {(0, 0): ec.source_key(*src[0]), (0, -1): ec.source_key(*src[-1])}
    assert ec.save_resident(eng, path, H, I, keys) == 2
    cache = ec.CacheFile(path)
    assert ec.make_resident(eng, cache, 0, 0, *src[0], H, I) is True          # cached, same source bytes
    assert ec.make_resident(eng, cache, 0, -1, *src[-1], H, I) is True        # the shared expert
    assert ec.make_resident(eng, cache, 0, 1, *src[1], H, I) is False         # not in the cache
    assert ec.make_resident(eng, cache, 0, 0, *src[1], H, I) is False         # other source bytes
    assert ec.make_resident(eng, cache, 0, 0, *src[0], H, I + 128) is False   # other shape
    assert ec.make_resident(eng, None, 0, 0, *src[0], H, I) is False
    cache.verify_all()
    assert ec.make_resident(eng, cache, 0, 0, *src[0], H, I, key=keys[(0, 0)], verify=False) is True
    assert ec.make_resident(eng, cache, 0, 0, *src[0], H, I, key=keys[(0, 0)] ^ 1, verify=False) is False
    assert eng.calls == [("import", 0, 0, bytes([0] * 4)), ("import", 0, -1, bytes([0xFF] * 4)),
                         ("upload", 0, 1), ("upload", 0, 0), ("upload", 0, 0), ("upload", 0, 0),
                         ("import", 0, 0, bytes([0] * 4)), ("upload", 0, 0)]


# -- the C reader of the same files (moe_b200_expert_cache_*, no device) -----

@pytest.fixture(scope="module")
def clib(pkg):
    import moe_b200.lib as L
    return L.load()


def _c_key(clib, g, u, d):
    import ctypes as C
    arrs = [np.ascontiguousarray(a, np.uint8) for a in (g, u, d)]
    ptr = lambda a: a.ctypes.data_as(C.c_void_p) if a.size else None
    return int(clib.moe_b200_source_key(ptr(arrs[0]), arrs[0].nbytes, ptr(arrs[1]), arrs[1].nbytes,
                                        ptr(arrs[2]), arrs[2].nbytes))


def test_c_source_key_matches_python(ec, clib):
    rng = np.random.default_rng(7)
    # lengths around the 128-byte BLAKE2b block, an empty part, a multi-block part
    for sizes in ((0, 0, 0), (1, 2, 3), (104, 0, 0), (120, 8, 0), (128, 128, 128), (127, 129, 256), (5000, 17, 1),
                  (170, 170, 340)):
        g, u, d = (rng.integers(0, 256, n, dtype=np.uint8) for n in sizes)
        assert _c_key(clib, g, u, d) == ec.source_key(g, u, d), sizes


def test_c_reader_matches_python_writer(ec, clib, tmp_path):
    import ctypes as C
    rng = np.random.default_rng(8)
    H, I = 256, 384
    recs = _records(ec, rng, H, I, [(0, 0), (0, 5), (0, -1), (3, 2)])
    path = str(tmp_path / "c.b200cache")
    ec.write_cache(path, H, I, recs)
    err = C.create_string_buffer(160)
    cache = clib.moe_b200_expert_cache_open(path.encode(), err)
    assert cache, err.value
    try:
        h, i, rb, n = C.c_uint32(), C.c_uint32(), C.c_uint64(), C.c_uint32()
        assert clib.moe_b200_expert_cache_info(cache, C.byref(h), C.byref(i), C.byref(rb), C.byref(n)) == 1
        assert (h.value, i.value, rb.value, n.value) == (H, I, ec.record_bytes(H, I), 4)
        for layer, expert, key, rec in recs:
            p = clib.moe_b200_expert_cache_record(cache, layer, expert, key, 1, err)
            assert p, err.value
            got = np.ctypeslib.as_array((C.c_uint8 * rb.value).from_address(p))
            assert np.array_equal(got, rec)
            # another source key or slot: no record, no error
            assert not clib.moe_b200_expert_cache_record(cache, layer, expert, key ^ 1, 1, err)
            assert err.value == b""
        assert not clib.moe_b200_expert_cache_record(cache, 1, 0, recs[0][2], 1, err)
    finally:
        clib.moe_b200_expert_cache_close(cache)
    # a flipped record byte: refused when checked, returned when not
    _corrupt(path, ec.CacheFile(path).entries[(0, 5)].offset + 99)
    cache = clib.moe_b200_expert_cache_open(path.encode(), err)
    assert cache, err.value
    try:
        assert not clib.moe_b200_expert_cache_record(cache, 0, 5, recs[1][2], 1, err)
        assert b"checksum" in err.value
        assert clib.moe_b200_expert_cache_record(cache, 0, 5, recs[1][2], 0, err)
        assert clib.moe_b200_expert_cache_record(cache, 0, 0, recs[0][2], 1, err)
    finally:
        clib.moe_b200_expert_cache_close(cache)
    # files the reader refuses: damaged table, wrong magic, truncated, absent
    for damage, msg in ((lambda: _corrupt(path, ec.HEADER_BYTES + 9), b"entry table checksum"),
                        (lambda: _corrupt(path, 1), b"not a repacked-expert cache"),
                        (lambda: open(path, "r+b").truncate(os.path.getsize(path) - ec.ALIGN), b"outside the file"),
                        (lambda: open(path, "r+b").truncate(64), b"shorter than the header")):
        ec.write_cache(path, H, I, recs)
        damage()
        assert not clib.moe_b200_expert_cache_open(path.encode(), err)
        assert msg in err.value, (msg, err.value)
    assert not clib.moe_b200_expert_cache_open(str(tmp_path / "absent").encode(), err)


def test_c_reader_survives_damaged_files(ec, clib, tmp_path):
    """Random byte flips anywhere in a cache file either leave it readable
    (the records still CRC-checked) or make open refuse it with a message;
    nothing is read outside the file."""
    import ctypes as C
    rng = np.random.default_rng(9)
    H, I = 128, 128
    recs = _records(ec, rng, H, I, [(0, 0), (0, 1), (1, 3)])
    clean = str(tmp_path / "clean.b200cache")
    ec.write_cache(clean, H, I, recs)
    data = bytearray(open(clean, "rb").read())
    err = C.create_string_buffer(160)
    path = str(tmp_path / "fuzz.b200cache")
    # header and entry table, where a flip changes what open believes
    spots = list(rng.integers(0, 64, 40)) + list(rng.integers(ec.HEADER_BYTES, ec.HEADER_BYTES + 3 * 64, 40))
    for off in spots:
        d = bytearray(data)
        d[int(off)] ^= int(rng.integers(1, 256))
        with open(path, "wb") as f:
            f.write(d)
        cache = clib.moe_b200_expert_cache_open(path.encode(), err)
        if not cache:
            assert err.value, off
            continue
        try:
            rb = C.c_uint64()
            assert clib.moe_b200_expert_cache_info(cache, None, None, C.byref(rb), None) == 1
            for layer, expert, key, rec in recs:
                p = clib.moe_b200_expert_cache_record(cache, layer, expert, key, 1, err)
                if p:  # a record that is returned is the one written
                    got = np.ctypeslib.as_array((C.c_uint8 * rb.value).from_address(p))
                    assert np.array_equal(got, rec)
        finally:
            clib.moe_b200_expert_cache_close(cache)
