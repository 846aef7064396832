"""Persisted repacked-expert cache: the engine's block-scaled expert records
in a file kept beside the model's JUJU sections.

The reference's residency upload (device_tensor_copy_ops.cpp.inc:73) copies
an expert's GGUF MXFP4 bytes to the device; this engine then repacks them into
the block-scaled layout its GEMMs read (moe_b200_upload_expert).  A cache file
keeps the repacked records, so an expert that becomes resident again is
installed with one plain copy (moe_b200_import_expert) and no repack, while
the JUJU file itself stays untouched: its payloads remain the source bytes.

Each record is keyed by (layer, expert) and by a 64-bit key of the source
bytes it was made from (source_key: BLAKE2b over the gate, up and down GGUF
bytes and their lengths).  A record whose key does not match the bytes the
caller is about to upload is not used, so a changed model cannot load stale
weights.  A CRC-32 of every record is checked when it is read.

File layout (little-endian):
  [0, 4096)       header: magic b"MOEB200R", version u32, header bytes u32,
                  hidden u32, intermediate u32, record bytes u64, entry count
                  u32, entry bytes u32 (64), entry table offset u64, CRC-32 of
                  the entry table u32; zero padding
  entry table     count x 64 bytes: layer i32, expert i32 (-1: shared
                  expert), source key u64, record offset u64, record CRC-32
                  u32; zero padding
  records         at 4096-aligned offsets, record bytes each
                  (moe_b200_expert_record_bytes(hidden, intermediate))
One file holds experts of one shape (H, I).
"""
from __future__ import annotations

import hashlib
import os
import struct
import zlib
from dataclasses import dataclass
from typing import Dict, Iterable, Optional, Tuple

import numpy as np

MAGIC = b"MOEB200R"
VERSION = 1
HEADER_BYTES = 4096
ENTRY_BYTES = 64
ALIGN = 4096
_HEADER = struct.Struct("<8sIIIIQIIQI")
_ENTRY = struct.Struct("<iiQQI")


class CacheError(RuntimeError):
    pass


def record_bytes(hidden: int, intermediate: int) -> int:
    """moe_b200_expert_record_bytes restated for the file layer (the host code
    that writes a cache needs no engine): four ranges with H and I padded to
    128 -- gate/up codes, gate/up scale blocks, down codes, down scale blocks."""
    if hidden <= 0 or intermediate <= 0 or hidden > 100000 or intermediate > 100000:
        return 0
    hp = -(-hidden // 128) * 128
    ip = -(-intermediate // 128) * 128
    return 2 * ip * (hp // 2) + 2 * (ip // 128) * (hp // 128) * 512 + hp * (ip // 2) + (hp // 128) * (ip // 128) * 512


def source_key(gate, up, down) -> int:
    """64-bit key of an expert's GGUF MXFP4 source bytes (gate, up, down)."""
    h = hashlib.blake2b(digest_size=8)
    for a in (gate, up, down):
        b = memoryview(np.ascontiguousarray(a)).cast("B")
        h.update(struct.pack("<Q", b.nbytes))
        h.update(b)
    return int.from_bytes(h.digest(), "little")


def _align(n: int) -> int:
    return -(-n // ALIGN) * ALIGN


@dataclass(frozen=True)
class Entry:
    layer: int
    expert: int
    key: int
    offset: int
    crc: int


def write_cache(path: str, hidden: int, intermediate: int,
                records: Iterable[Tuple[int, int, int, np.ndarray]]) -> int:
    """Writes (layer, expert, source key, record bytes) tuples to `path`
    (replaced atomically); returns the number of records."""
    rb = record_bytes(hidden, intermediate)
    if rb == 0:
        raise CacheError(f"no expert record for H={hidden} I={intermediate}")
    items = []
    seen = set()
    for layer, expert, key, rec in records:
        rec = np.ascontiguousarray(rec).view(np.uint8).reshape(-1)
        if rec.nbytes != rb:
            raise CacheError(f"record of layer {layer} expert {expert} is {rec.nbytes} bytes, expected {rb}")
        if (layer, expert) in seen:
            raise CacheError(f"layer {layer} expert {expert} given twice")
        seen.add((layer, expert))
        items.append((int(layer), int(expert), int(key) & (2**64 - 1), rec))
    table_off = HEADER_BYTES
    data_off = _align(table_off + ENTRY_BYTES * len(items))
    stride = _align(rb)
    table = bytearray(ENTRY_BYTES * len(items))
    for i, (layer, expert, key, rec) in enumerate(items):
        _ENTRY.pack_into(table, i * ENTRY_BYTES, layer, expert, key, data_off + i * stride, zlib.crc32(rec))
    header = bytearray(HEADER_BYTES)
    _HEADER.pack_into(header, 0, MAGIC, VERSION, HEADER_BYTES, hidden, intermediate, rb, len(items), ENTRY_BYTES,
                      table_off, zlib.crc32(table))
    tmp = f"{path}.tmp{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(header)
        f.write(table)
        f.write(b"\0" * (data_off - table_off - len(table)))
        for _, _, _, rec in items:
            f.write(rec.tobytes())
            f.write(b"\0" * (stride - rb))
    os.replace(tmp, path)
    return len(items)


class CacheFile:
    """A cache file opened read-only (memory-mapped records)."""

    def __init__(self, path: str):
        size = os.path.getsize(path)
        if size < HEADER_BYTES:
            raise CacheError(f"{path}: {size} bytes, shorter than the header")
        with open(path, "rb") as f:
            head = f.read(HEADER_BYTES)
            (magic, version, hbytes, self.hidden, self.intermediate, self.record_bytes, count, ebytes, table_off,
             table_crc) = _HEADER.unpack_from(head, 0)
            if magic != MAGIC:
                raise CacheError(f"{path}: not a repacked-expert cache")
            if version != VERSION or hbytes != HEADER_BYTES or ebytes != ENTRY_BYTES:
                raise CacheError(f"{path}: version {version} / header {hbytes} / entry {ebytes} not supported")
            if self.record_bytes != record_bytes(self.hidden, self.intermediate):
                raise CacheError(f"{path}: record size {self.record_bytes} does not match H={self.hidden} "
                                 f"I={self.intermediate}")
            if table_off + count * ENTRY_BYTES > size:
                raise CacheError(f"{path}: entry table past the end of the file")
            f.seek(table_off)
            table = f.read(count * ENTRY_BYTES)
        if zlib.crc32(table) != table_crc:
            raise CacheError(f"{path}: entry table checksum mismatch")
        self.path = path
        self.entries: Dict[Tuple[int, int], Entry] = {}
        for i in range(count):
            layer, expert, key, off, crc = _ENTRY.unpack_from(table, i * ENTRY_BYTES)
            if off % ALIGN or off + self.record_bytes > size:
                raise CacheError(f"{path}: record of layer {layer} expert {expert} outside the file")
            self.entries[(layer, expert)] = Entry(layer, expert, key, off, crc)
        self._map = np.memmap(path, np.uint8, mode="r") if count else None

    def get(self, layer: int, expert: int, key: Optional[int] = None, verify: bool = True) -> Optional[np.ndarray]:
        """The record of (layer, expert), checked against its CRC unless
        verify is False (after verify_all); None when the file has none or its
        source key differs from `key`."""
        e = self.entries.get((layer, expert))
        if e is None or (key is not None and e.key != (int(key) & (2**64 - 1))):
            return None
        rec = np.asarray(self._map[e.offset:e.offset + self.record_bytes])
        if verify and zlib.crc32(rec) != e.crc:
            raise CacheError(f"{self.path}: record of layer {layer} expert {expert} fails its checksum")
        return rec

    def verify_all(self):
        """Checks every record's CRC once (e.g. when the cache is opened), so
        that residency events can read records with verify=False."""
        for (layer, expert) in self.entries:
            self.get(layer, expert)

    def close(self):
        self._map = None


def save_resident(engine, path: str, hidden: int, intermediate: int, keys: Dict[Tuple[int, int], int]) -> int:
    """Exports the engine's resident experts named in `keys` ((layer, expert)
    -> source key) into a cache file at `path`."""
    recs = ((layer, expert, key, engine.export_expert(layer, expert, hidden, intermediate))
            for (layer, expert), key in sorted(keys.items()))
    return write_cache(path, hidden, intermediate, recs)


def make_resident(engine, cache: Optional[CacheFile], layer: int, expert: int, gate, up, down, hidden: int,
                  intermediate: int, key: Optional[int] = None, verify: bool = True) -> bool:
    """Makes one expert resident: from its cached record when the cache holds
    one made from these source bytes (no repack; returns True), else by the
    repacking upload (returns False).  `key`: the source key if the caller
    keeps it (a residency index computes it once per model), else it is
    computed from the bytes here; `verify`: CacheFile.get's record check."""
    if cache is not None and cache.hidden == hidden and cache.intermediate == intermediate:
        rec = cache.get(layer, expert, source_key(gate, up, down) if key is None else key, verify=verify)
        if rec is not None:
            engine.import_expert(layer, expert, rec, hidden, intermediate)
            return True
    engine.upload_expert(layer, expert, np.ascontiguousarray(gate), np.ascontiguousarray(up),
                         np.ascontiguousarray(down), hidden, intermediate)
    return False
