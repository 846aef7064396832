// Repacked-expert cache files read from C (host code only): the same file
// that storage.llm_b200/expert_cache.py writes, so an engine written in C or
// C++ (the reference's residency hook, device_tensor_copy_ops.cpp.inc:73) can
// find a cached record and install it with moe_b200_import_expert.
//
// File layout (little-endian): a 4096-byte header -- magic "MOEB200R",
// version 1, header bytes, hidden, intermediate, record bytes, entry count,
// entry bytes (64), entry table offset, CRC-32 of the entry table -- then
// 64-byte entries (layer, expert, source key, record offset, record CRC-32),
// then the records at 4096-aligned offsets.
//
// Source keys are BLAKE2b with an 8-byte digest (RFC 7693, no key) over, for
// each of gate, up and down: the byte count as 8 little-endian bytes, then
// the bytes.  CRC-32 is the zlib one (reflected polynomial 0xEDB88320).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <new>
#include <unordered_map>

#include "../../include/moe_b200.h"
#include "engine.h"

namespace {

using moe_b200::set_err;

// ---------------------------------------------------------------- BLAKE2b
// RFC 7693: 64-bit words, 12 rounds, G rotations 32/24/16/63, the SHA-512
// initial values, the message schedule SIGMA (rounds 10 and 11 reuse rows 0
// and 1).
constexpr uint64_t kIv[8] = {0x6a09e667f3bcc908ull, 0xbb67ae8584caa73bull, 0x3c6ef372fe94f82bull,
                             0xa54ff53a5f1d36f1ull, 0x510e527fade682d1ull, 0x9b05688c2b3e6c1full,
                             0x1f83d9abfb41bd6bull, 0x5be0cd19137e2179ull};
constexpr uint8_t kSigma[10][16] = {
    {0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15}, {14, 10, 4, 8, 9, 15, 13, 6, 1, 12, 0, 2, 11, 7, 5, 3},
    {11, 8, 12, 0, 5, 2, 15, 13, 10, 14, 3, 6, 7, 1, 9, 4}, {7, 9, 3, 1, 13, 12, 11, 14, 2, 6, 5, 10, 4, 0, 15, 8},
    {9, 0, 5, 7, 2, 4, 10, 15, 14, 1, 11, 12, 6, 8, 3, 13}, {2, 12, 6, 10, 0, 11, 8, 3, 4, 13, 7, 5, 15, 14, 1, 9},
    {12, 5, 1, 15, 14, 13, 4, 10, 0, 7, 6, 3, 9, 2, 8, 11}, {13, 11, 7, 14, 12, 1, 3, 9, 5, 0, 15, 4, 8, 6, 2, 10},
    {6, 15, 14, 9, 11, 3, 0, 8, 12, 2, 13, 7, 1, 4, 10, 5}, {10, 2, 8, 4, 7, 6, 1, 5, 15, 11, 9, 14, 3, 12, 13, 0}};

inline uint64_t rotr64(uint64_t x, int n) { return (x >> n) | (x << (64 - n)); }

inline uint64_t load_le64(const uint8_t* p) {
    uint64_t v = 0;
    for (int i = 7; i >= 0; --i) v = (v << 8) | p[i];
    return v;
}

struct Blake2b {
    uint64_t h[8];
    uint64_t t0 = 0, t1 = 0;  // bytes compressed so far (128-bit counter)
    uint8_t buf[128];
    size_t fill = 0;
    size_t outlen;

    explicit Blake2b(size_t out) : outlen(out) {
        for (int i = 0; i < 8; ++i) h[i] = kIv[i];
        h[0] ^= 0x01010000ull ^ (uint64_t)out;  // fanout 1, depth 1, no key
    }

    void compress(const uint8_t* block, bool last) {
        uint64_t m[16], v[16];
        for (int i = 0; i < 16; ++i) m[i] = load_le64(block + 8 * i);
        for (int i = 0; i < 8; ++i) {
            v[i] = h[i];
            v[i + 8] = kIv[i];
        }
        v[12] ^= t0;
        v[13] ^= t1;
        if (last) v[14] = ~v[14];
        auto g = [&](int a, int b, int c, int d, uint64_t x, uint64_t y) {
            v[a] = v[a] + v[b] + x;
            v[d] = rotr64(v[d] ^ v[a], 32);
            v[c] = v[c] + v[d];
            v[b] = rotr64(v[b] ^ v[c], 24);
            v[a] = v[a] + v[b] + y;
            v[d] = rotr64(v[d] ^ v[a], 16);
            v[c] = v[c] + v[d];
            v[b] = rotr64(v[b] ^ v[c], 63);
        };
        for (int r = 0; r < 12; ++r) {
            const uint8_t* s = kSigma[r % 10];
            g(0, 4, 8, 12, m[s[0]], m[s[1]]);
            g(1, 5, 9, 13, m[s[2]], m[s[3]]);
            g(2, 6, 10, 14, m[s[4]], m[s[5]]);
            g(3, 7, 11, 15, m[s[6]], m[s[7]]);
            g(0, 5, 10, 15, m[s[8]], m[s[9]]);
            g(1, 6, 11, 12, m[s[10]], m[s[11]]);
            g(2, 7, 8, 13, m[s[12]], m[s[13]]);
            g(3, 4, 9, 14, m[s[14]], m[s[15]]);
        }
        for (int i = 0; i < 8; ++i) h[i] ^= v[i] ^ v[i + 8];
    }

    void count(size_t n) {
        t0 += n;
        if (t0 < n) ++t1;
    }

    // a full buffer is compressed only once more input follows (the last
    // block must be compressed with the final flag)
    void update(const uint8_t* p, size_t n) {
        while (n > 0) {
            if (fill == sizeof(buf)) {
                count(sizeof(buf));
                compress(buf, false);
                fill = 0;
            }
            const size_t take = n < sizeof(buf) - fill ? n : sizeof(buf) - fill;
            std::memcpy(buf + fill, p, take);
            fill += take;
            p += take;
            n -= take;
        }
    }

    void finish(uint8_t* out) {
        count(fill);
        std::memset(buf + fill, 0, sizeof(buf) - fill);
        compress(buf, true);
        for (size_t i = 0; i < outlen; ++i) out[i] = (uint8_t)(h[i / 8] >> (8 * (i % 8)));
    }
};

// ---------------------------------------------------------------- CRC-32
struct CrcTable {
    uint32_t v[256];
    CrcTable() {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c & 1u) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
            v[i] = c;
        }
    }
};

uint32_t crc32(const uint8_t* p, uint64_t n) {
    static const CrcTable tab;  // initialised once, thread-safely
    const uint32_t* table = tab.v;
    uint32_t c = 0xFFFFFFFFu;
    for (uint64_t i = 0; i < n; ++i) c = table[(c ^ p[i]) & 0xFFu] ^ (c >> 8);
    return c ^ 0xFFFFFFFFu;
}

inline uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }

constexpr uint64_t kHeaderBytes = 4096, kEntryBytes = 64, kAlign = 4096;

struct Entry {
    uint64_t key, offset;
    uint32_t crc;
};

}  // namespace

struct moe_b200_expert_cache {
    void* map = nullptr;
    uint64_t size = 0;
    uint32_t hidden = 0, intermediate = 0, entries = 0;
    uint64_t record_bytes = 0;
    std::unordered_map<uint64_t, Entry> index;  // (layer, expert) -> entry
};

namespace {

uint64_t slot_key(int32_t layer, int32_t expert) { return (uint64_t)(uint32_t)layer << 32 | (uint32_t)expert; }

}  // namespace

extern "C" {

uint64_t moe_b200_source_key(const uint8_t* gate, uint64_t gate_bytes, const uint8_t* up, uint64_t up_bytes,
                             const uint8_t* down, uint64_t down_bytes) {
    Blake2b b(8);
    const uint8_t* parts[3] = {gate, up, down};
    const uint64_t sizes[3] = {gate_bytes, up_bytes, down_bytes};
    for (int i = 0; i < 3; ++i) {
        uint8_t len[8];
        for (int j = 0; j < 8; ++j) len[j] = (uint8_t)(sizes[i] >> (8 * j));
        b.update(len, 8);
        if (sizes[i]) b.update(parts[i], sizes[i]);
    }
    uint8_t out[8];
    b.finish(out);
    return load_le64(out);
}

moe_b200_expert_cache_t* moe_b200_expert_cache_open(const char* path, char* err) {
    if (!path) {
        set_err(err, "null path");
        return nullptr;
    }
    const int fd = open(path, O_RDONLY);
    if (fd < 0) {
        set_err(err, "%s: cannot open", path);
        return nullptr;
    }
    struct stat st {};
    if (fstat(fd, &st) != 0 || (uint64_t)st.st_size < kHeaderBytes) {
        close(fd);
        set_err(err, "%s: shorter than the header", path);
        return nullptr;
    }
    const uint64_t size = (uint64_t)st.st_size;
    void* map = mmap(nullptr, size, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (map == MAP_FAILED) {
        set_err(err, "%s: mmap failed", path);
        return nullptr;
    }
    const uint8_t* b = static_cast<const uint8_t*>(map);
    auto fail = [&](const char* what) -> moe_b200_expert_cache_t* {
        munmap(map, size);
        set_err(err, "%s: %s", path, what);
        return nullptr;
    };
    if (std::memcmp(b, "MOEB200R", 8) != 0) return fail("not a repacked-expert cache");
    const uint32_t version = rd32(b + 8), hbytes = rd32(b + 12), hidden = rd32(b + 16), inter = rd32(b + 20);
    const uint64_t rbytes = load_le64(b + 24);
    const uint32_t count = rd32(b + 32), ebytes = rd32(b + 36);
    const uint64_t table_off = load_le64(b + 40);
    const uint32_t table_crc = rd32(b + 48);
    if (version != 1 || hbytes != kHeaderBytes || ebytes != kEntryBytes) return fail("version or layout not supported");
    if (rbytes == 0 || rbytes != moe_b200_expert_record_bytes(hidden, inter)) {
        return fail("record size does not match its H and I");
    }
    if (table_off > size || (uint64_t)count * kEntryBytes > size - table_off) {
        return fail("entry table past the end of the file");
    }
    if (crc32(b + table_off, (uint64_t)count * kEntryBytes) != table_crc) return fail("entry table checksum mismatch");
    auto* c = new (std::nothrow) moe_b200_expert_cache();
    if (!c) return fail("out of host memory");
    for (uint32_t i = 0; i < count; ++i) {
        const uint8_t* e = b + table_off + (uint64_t)i * kEntryBytes;
        const int32_t layer = (int32_t)rd32(e), expert = (int32_t)rd32(e + 4);
        Entry en{load_le64(e + 8), load_le64(e + 16), rd32(e + 24)};
        if (en.offset % kAlign || en.offset > size || rbytes > size - en.offset) {
            delete c;
            return fail("a record lies outside the file");
        }
        c->index[slot_key(layer, expert)] = en;
    }
    c->map = map;
    c->size = size;
    c->hidden = hidden;
    c->intermediate = inter;
    c->record_bytes = rbytes;
    c->entries = count;
    return c;
}

void moe_b200_expert_cache_close(moe_b200_expert_cache_t* cache) {
    if (!cache) return;
    if (cache->map) munmap(cache->map, cache->size);
    delete cache;
}

int moe_b200_expert_cache_info(const moe_b200_expert_cache_t* cache, uint32_t* hidden, uint32_t* intermediate,
                               uint64_t* record_bytes, uint32_t* entries) {
    if (!cache) return 0;
    if (hidden) *hidden = cache->hidden;
    if (intermediate) *intermediate = cache->intermediate;
    if (record_bytes) *record_bytes = cache->record_bytes;
    if (entries) *entries = cache->entries;
    return 1;
}

const uint8_t* moe_b200_expert_cache_record(const moe_b200_expert_cache_t* cache, int32_t layer, int32_t expert,
                                            uint64_t source_key, int32_t verify, char* err) {
    if (err) err[0] = 0;
    if (!cache) {
        set_err(err, "null cache");
        return nullptr;
    }
    const auto it = cache->index.find(slot_key(layer, expert));
    if (it == cache->index.end() || it->second.key != source_key) return nullptr;
    const uint8_t* rec = static_cast<const uint8_t*>(cache->map) + it->second.offset;
    if (verify && crc32(rec, cache->record_bytes) != it->second.crc) {
        set_err(err, "record of layer %d expert %d fails its checksum", layer, expert);
        return nullptr;
    }
    return rec;
}

}  // extern "C"
