// nt_checkpoint.cu -- the on-disk format: named, typed, checksummed sections (host code).
//
// The reference keeps no training state on disk (its driver writes EXR images,
// mavenkim2/neural_textures main.cpp:855-904).  Layout, little-endian:
//   0    "NTB2CKPT"
//   8    u32 version (1), u32 section count
//   16   u64 index offset, u64 FNV-1a 64 of the index
//   32   zero up to 64
//   64   payloads, each at a 64-byte aligned offset (zero padding between them)
//   ...  index: per section name[32], i32 dtype, i32 ndim, i64 shape[4], u64 offset, u64 bytes,
//        u64 FNV-1a 64 of the payload
// FNV-1a 64 (Fowler, Noll, Vo: offset basis 14695981039346656037, prime 1099511628211).
#include <fcntl.h>
#include <unistd.h>

#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "nt_capi.h"

namespace nt {

nt_status set_error(nt_status st, const char *fmt, ...);

namespace {

constexpr char kMagic[8] = {'N', 'T', 'B', '2', 'C', 'K', 'P', 'T'};
constexpr uint32_t kVersion = 1;
constexpr uint64_t kAlign = 64;

struct Entry {
    char name[NT_CKPT_NAME_LEN];
    int32_t dtype;
    int32_t ndim;
    int64_t shape[4];
    uint64_t offset;
    uint64_t bytes;
    uint64_t checksum;
};
static_assert(sizeof(Entry) == 96, "index entry layout");

struct Header {
    char magic[8];
    uint32_t version;
    uint32_t count;
    uint64_t index_offset;
    uint64_t index_checksum;
    uint8_t pad[32];
};
static_assert(sizeof(Header) == 64, "header layout");

uint64_t fnv1a(const void *data, uint64_t n, uint64_t h = 14695981039346656037ull)
{
    const uint8_t *p = static_cast<const uint8_t *>(data);
    for (uint64_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}

int64_t dtype_size(int32_t dt)
{
    switch (dt) {
    case NT_DTYPE_F16: return 2;
    case NT_DTYPE_F32: return 4;
    case NT_DTYPE_U8: return 1;
    case NT_DTYPE_I32: return 4;
    default: return 0;
    }
}

struct File {
    FILE *f = nullptr;
    ~File()
    {
        if (f) fclose(f);
    }
};

bool valid_name(const char *name)
{
    const size_t n = strnlen(name, NT_CKPT_NAME_LEN);
    return n > 0 && n < NT_CKPT_NAME_LEN;
}

nt_status check_section(const NtCheckpointSection &s, int i)
{
    if (!valid_name(s.name)) return set_error(NT_ERR_INVALID_ARG, "section %d: name must be 1 .. %d characters", i, NT_CKPT_NAME_LEN - 1);
    const int64_t es = dtype_size(s.dtype);
    if (es == 0) return set_error(NT_ERR_INVALID_ARG, "section '%s': unknown dtype %d", s.name, s.dtype);
    if (s.ndim < 0 || s.ndim > 4) return set_error(NT_ERR_INVALID_ARG, "section '%s': ndim must be 0 .. 4", s.name);
    int64_t n = 1;
    for (int d = 0; d < s.ndim; ++d) {
        if (s.shape[d] < 0 || (s.shape[d] > 0 && n > INT64_MAX / 8 / s.shape[d]))
            return set_error(NT_ERR_INVALID_ARG, "section '%s': bad shape", s.name);
        n *= s.shape[d];
    }
    if (s.bytes != n * es)
        return set_error(NT_ERR_INVALID_ARG, "section '%s': bytes %lld do not match its shape (%lld)", s.name,
                         (long long)s.bytes, (long long)(n * es));
    return NT_OK;
}

// Header and index of an open file (checked against the file size and the index checksum).
nt_status load_index(FILE *f, const char *path, std::vector<Entry> &entries)
{
    Header h;
    if (fseek(f, 0, SEEK_END) != 0) return set_error(NT_ERR_IO, "%s: cannot seek", path);
    const long size = ftell(f);
    if (size < (long)sizeof(Header) || fseek(f, 0, SEEK_SET) != 0 || fread(&h, sizeof h, 1, f) != 1)
        return set_error(NT_ERR_IO, "%s: truncated header", path);
    if (memcmp(h.magic, kMagic, 8) != 0) return set_error(NT_ERR_IO, "%s: not a checkpoint file", path);
    if (h.version != kVersion)
        return set_error(NT_ERR_IO, "%s: checkpoint version %u (this library reads %u)", path, h.version, kVersion);
    if (h.count > NT_CKPT_MAX_SECTIONS) return set_error(NT_ERR_IO, "%s: %u sections", path, h.count);
    const uint64_t ibytes = (uint64_t)h.count * sizeof(Entry);
    if (h.index_offset < sizeof(Header) || h.index_offset + ibytes != (uint64_t)size)
        return set_error(NT_ERR_IO, "%s: truncated or corrupt index", path);
    entries.resize(h.count);
    if (h.count && (fseek(f, (long)h.index_offset, SEEK_SET) != 0 || fread(entries.data(), sizeof(Entry), h.count, f) != h.count))
        return set_error(NT_ERR_IO, "%s: cannot read the index", path);
    if (fnv1a(entries.data(), ibytes) != h.index_checksum) return set_error(NT_ERR_IO, "%s: index checksum mismatch", path);
    for (const Entry &e : entries)
        if (!valid_name(e.name) || e.offset < sizeof(Header) || e.offset + e.bytes > h.index_offset)
            return set_error(NT_ERR_IO, "%s: corrupt index entry", path);
    return NT_OK;
}

}  // namespace
}  // namespace nt

using namespace nt;

extern "C" {

nt_status nt_checkpoint_write(const char *path, const NtCheckpointSection *sections, int32_t count)
{
    if (!path || !*path) return set_error(NT_ERR_INVALID_ARG, "path is empty");
    if (count < 0 || count > NT_CKPT_MAX_SECTIONS || (count > 0 && !sections))
        return set_error(NT_ERR_INVALID_ARG, "section count must be in [0, %d]", NT_CKPT_MAX_SECTIONS);
    for (int i = 0; i < count; ++i) {
        nt_status st = check_section(sections[i], i);
        if (st != NT_OK) return st;
        if (sections[i].bytes > 0 && !sections[i].data)
            return set_error(NT_ERR_INVALID_ARG, "section '%s': data is null", sections[i].name);
        for (int j = 0; j < i; ++j)
            if (strncmp(sections[i].name, sections[j].name, NT_CKPT_NAME_LEN) == 0)
                return set_error(NT_ERR_INVALID_ARG, "section name '%s' is used twice", sections[i].name);
    }
    const std::string tmp = std::string(path) + ".tmp";
    std::vector<Entry> entries((size_t)count);
    // The file is written to path + ".tmp", flushed to the device, then renamed over path
    // and the directory entry flushed too, so that a crash leaves either the old file or the
    // new one.  A failed write removes the .tmp file.
    const auto write_tmp = [&]() -> nt_status {
        File out;
        out.f = fopen(tmp.c_str(), "wb");
        if (!out.f) return set_error(NT_ERR_IO, "%s: cannot create (%s)", tmp.c_str(), strerror(errno));
        Header h;
        memset(&h, 0, sizeof h);
        if (fwrite(&h, sizeof h, 1, out.f) != 1) return set_error(NT_ERR_IO, "%s: write failed", tmp.c_str());
        uint64_t pos = sizeof h;
        static const uint8_t zeros[kAlign] = {};
        for (int i = 0; i < count; ++i) {
            const NtCheckpointSection &s = sections[i];
            const uint64_t pad = (kAlign - pos % kAlign) % kAlign;
            if (pad && fwrite(zeros, 1, pad, out.f) != pad) return set_error(NT_ERR_IO, "%s: write failed", tmp.c_str());
            pos += pad;
            Entry &e = entries[(size_t)i];
            memset(&e, 0, sizeof e);
            strncpy(e.name, s.name, NT_CKPT_NAME_LEN - 1);
            e.dtype = s.dtype;
            e.ndim = s.ndim;
            for (int d = 0; d < 4; ++d) e.shape[d] = d < s.ndim ? s.shape[d] : 0;
            e.offset = pos;
            e.bytes = (uint64_t)s.bytes;
            e.checksum = fnv1a(s.data, e.bytes);
            if (e.bytes && fwrite(s.data, 1, e.bytes, out.f) != e.bytes)
                return set_error(NT_ERR_IO, "%s: write failed", tmp.c_str());
            pos += e.bytes;
        }
        h.index_offset = pos;
        if (count && fwrite(entries.data(), sizeof(Entry), (size_t)count, out.f) != (size_t)count)
            return set_error(NT_ERR_IO, "%s: write failed", tmp.c_str());
        memcpy(h.magic, kMagic, 8);
        h.version = kVersion;
        h.count = (uint32_t)count;
        h.index_checksum = fnv1a(entries.data(), (uint64_t)count * sizeof(Entry));
        if (fseek(out.f, 0, SEEK_SET) != 0 || fwrite(&h, sizeof h, 1, out.f) != 1 || fflush(out.f) != 0)
            return set_error(NT_ERR_IO, "%s: write failed", tmp.c_str());
        if (fsync(fileno(out.f)) != 0) return set_error(NT_ERR_IO, "%s: fsync failed (%s)", tmp.c_str(), strerror(errno));
        const int rc = fclose(out.f);
        out.f = nullptr;
        if (rc != 0) return set_error(NT_ERR_IO, "%s: close failed", tmp.c_str());
        return NT_OK;
    };
    nt_status st = write_tmp();
    if (st != NT_OK) {
        remove(tmp.c_str());
        return st;
    }
    if (rename(tmp.c_str(), path) != 0) {
        const int err = errno;
        remove(tmp.c_str());
        return set_error(NT_ERR_IO, "%s: rename failed (%s)", path, strerror(err));
    }
    {  // flush the directory entry of the rename
        std::string dir(path);
        const size_t slash = dir.find_last_of('/');
        dir = slash == std::string::npos ? std::string(".") : (slash == 0 ? std::string("/") : dir.substr(0, slash));
        const int fd = open(dir.c_str(), O_RDONLY | O_DIRECTORY);
        if (fd >= 0) {
            fsync(fd);
            close(fd);
        }
    }
    return NT_OK;
}

nt_status nt_checkpoint_index(const char *path, NtCheckpointSection *sections, int32_t capacity, int32_t *count)
{
    if (!path || !count) return set_error(NT_ERR_INVALID_ARG, "path and count are required");
    if (capacity < 0 || (capacity > 0 && !sections)) return set_error(NT_ERR_INVALID_ARG, "bad capacity");
    File in;
    in.f = fopen(path, "rb");
    if (!in.f) return set_error(NT_ERR_IO, "%s: cannot open (%s)", path, strerror(errno));
    std::vector<Entry> entries;
    nt_status st = load_index(in.f, path, entries);
    if (st != NT_OK) return st;
    *count = (int32_t)entries.size();
    if (capacity > 0 && capacity < (int32_t)entries.size())
        return set_error(NT_ERR_INVALID_ARG, "%s holds %d sections, capacity is %d", path, (int)entries.size(), capacity);
    for (int i = 0; i < (int)entries.size() && i < capacity; ++i) {
        NtCheckpointSection &s = sections[i];
        memset(&s, 0, sizeof s);
        memcpy(s.name, entries[(size_t)i].name, NT_CKPT_NAME_LEN);
        s.dtype = entries[(size_t)i].dtype;
        s.ndim = entries[(size_t)i].ndim;
        for (int d = 0; d < 4; ++d) s.shape[d] = entries[(size_t)i].shape[d];
        s.bytes = (int64_t)entries[(size_t)i].bytes;
    }
    return NT_OK;
}

nt_status nt_checkpoint_read(const char *path, const char *name, void *dst, int64_t bytes)
{
    if (!path || !name) return set_error(NT_ERR_INVALID_ARG, "path and name are required");
    if (bytes < 0 || (bytes > 0 && !dst)) return set_error(NT_ERR_INVALID_ARG, "bad destination");
    File in;
    in.f = fopen(path, "rb");
    if (!in.f) return set_error(NT_ERR_IO, "%s: cannot open (%s)", path, strerror(errno));
    std::vector<Entry> entries;
    nt_status st = load_index(in.f, path, entries);
    if (st != NT_OK) return st;
    for (const Entry &e : entries) {
        if (strncmp(e.name, name, NT_CKPT_NAME_LEN) != 0) continue;
        if ((uint64_t)bytes != e.bytes)
            return set_error(NT_ERR_INVALID_ARG, "section '%s' holds %llu bytes, the destination %lld", name,
                             (unsigned long long)e.bytes, (long long)bytes);
        if (e.bytes && (fseek(in.f, (long)e.offset, SEEK_SET) != 0 || fread(dst, 1, e.bytes, in.f) != e.bytes))
            return set_error(NT_ERR_IO, "%s: cannot read section '%s'", path, name);
        if (fnv1a(dst, e.bytes) != e.checksum) return set_error(NT_ERR_IO, "%s: section '%s' checksum mismatch", path, name);
        return NT_OK;
    }
    return set_error(NT_ERR_INVALID_ARG, "%s has no section '%s'", path, name);
}

}  // extern "C"
