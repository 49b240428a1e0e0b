// safetensors.cpp -- the validating, memory-mapped safetensors reader (the counterpart of SafetensorsFile,
// src/Lrm.Tensor/Safetensors.fs:231-727) behind the lrm_st_* entry points.
//
// A file is 8 bytes of little-endian header length N, N bytes of UTF-8 JSON, then the data section. Open maps the
// file read-only and checks, before anything is returned, the rules of SafetensorsParse.header (Safetensors.fs:297-
// 500): N <= 100,000,000 and within the file; the header starts with '{' and is valid UTF-8 (no overlong forms, no
// encoded surrogates) and valid JSON of depth <= 8 whose \u escapes form valid Unicode; no duplicate key at any
// level; "__metadata__" is an object of strings; every other key is a non-empty tensor name whose value has exactly
// the fields dtype (F32, F64, BF16, F16, I32, U32, U8, I64), shape (non-negative integers) and data_offsets (a pair of
// non-negative integers) with end - begin = elements x element size and end within the data section; and the tensors
// tile the data section exactly (no hole, no overlap, nothing after the last one). Entries and metadata are kept in
// code point order of their names (byte order of UTF-8). Messages name the file.
#include <errno.h>
#include <fcntl.h>
#include <stdint.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <memory>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/lrm_cuda.h"
#include "internal.h"
#include "json.h"
#include "safetensors.h"

namespace lrm {
namespace st {

namespace {

constexpr uint64_t kMaxHeaderBytes = 100000000ull;
constexpr int kMaxDepth = 8;
using json::JValue;
using json::valid_utf8;

struct FormatError {
    std::string msg;
};

[[noreturn]] void fail(const std::string &m) { throw FormatError{m}; }

const char *const kDtypeNames[] = {"F32", "F64", "BF16", "F16", "I32", "U32", "U8", "I64"};
const int kDtypeSizes[] = {4, 8, 2, 2, 4, 4, 1, 8};

// A non-negative JSON integer (digits only, as System.Text.Json's TryGetInt64 accepts; no sign, fraction or
// exponent) within int64.
int64_t non_negative(const std::string &where, const JValue &v) {
    if (v.kind != JValue::NUMBER) fail(where + " is not a non-negative integer");
    const std::string &t = v.text;
    if (t.empty() || t.size() > 19) fail(where + " is not a non-negative integer");
    int64_t x = 0;
    for (char c : t) {
        if (c < '0' || c > '9') fail(where + " is not a non-negative integer");
        x = x * 10 + (c - '0');
    }
    if (t.size() == 19 && t > "9223372036854775807") fail(where + " is not a non-negative integer");
    return x;
}

Entry entry(uint64_t data_len, const std::string &name, const JValue &v) {
    if (name.empty()) fail("empty tensor name");
    if (v.kind != JValue::OBJECT) fail(name + ": the entry is not an object");
    int dtype = -1;
    bool have_shape = false, have_offsets = false;
    std::vector<int64_t> shape;
    uint64_t b = 0, e = 0;
    std::vector<std::string> seen;
    for (const auto &m : v.members) {
        const std::string &f = m.first;
        if (std::find(seen.begin(), seen.end(), f) != seen.end()) fail(name + ": duplicate field '" + f + "'");
        seen.push_back(f);
        if (f == "dtype") {
            if (m.second.kind != JValue::STRING) fail(name + ": dtype is not a string");
            for (int d = 0; d < 8; ++d)
                if (m.second.text == kDtypeNames[d]) dtype = d;
            if (dtype < 0) fail(name + ": unsupported dtype '" + m.second.text + "'");
        } else if (f == "shape") {
            if (m.second.kind != JValue::ARRAY) fail(name + ": shape is not an array");
            for (const auto &d : m.second.items) shape.push_back(non_negative(name + ": shape", d));
            have_shape = true;
        } else if (f == "data_offsets") {
            if (m.second.kind != JValue::ARRAY || m.second.items.size() != 2) fail(name + ": data_offsets is not a pair");
            b = (uint64_t)non_negative(name + ": data_offsets", m.second.items[0]);
            e = (uint64_t)non_negative(name + ": data_offsets", m.second.items[1]);
            have_offsets = true;
        } else {
            fail(name + ": unknown field '" + f + "'");
        }
    }
    if (dtype < 0 || !have_shape || !have_offsets) fail(name + ": the entry needs dtype, shape and data_offsets");
    unsigned __int128 elems = 1;
    for (int64_t d : shape) {
        elems *= (uint64_t)d;
        if (elems > (unsigned __int128)INT64_MAX) fail(name + ": the byte count overflows");
    }
    const unsigned __int128 bytes = elems * (unsigned)kDtypeSizes[dtype];
    if (bytes > (unsigned __int128)INT64_MAX) fail(name + ": the byte count overflows");
    if (e < b) fail(name + ": data_offsets [" + std::to_string(b) + ", " + std::to_string(e) + "] are reversed");
    if ((unsigned __int128)(e - b) != bytes)
        fail(name + ": " + std::to_string(e - b) + " bytes for " + kDtypeNames[dtype] + " (expected " +
             std::to_string((uint64_t)bytes) + ")");
    if (e > data_len)
        fail(name + ": data_offsets end " + std::to_string(e) + " is beyond the data section (" +
             std::to_string(data_len) + " bytes)");
    Entry out;
    out.name = name;
    out.dtype = dtype;
    out.shape = std::move(shape);
    out.begin = b;
    out.end = e;
    return out;
}

}  // namespace

void parse(const uint8_t *bytes, uint64_t length, Parsed &out) {
    if (length < 8) fail(std::to_string(length) + " bytes is shorter than the 8-byte header length");
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | bytes[i];
    if (n > kMaxHeaderBytes) fail("header length " + std::to_string(n) + " exceeds 100000000");
    if (n > length - 8) fail("header length " + std::to_string(n) + " exceeds the file (" + std::to_string(length) + " bytes)");
    const uint64_t data_len = length - 8 - n;
    const uint8_t *h = bytes + 8;
    if (n == 0 || h[0] != '{') fail("the header is not a JSON object");
    if (!valid_utf8(h, n)) fail("the header is not valid UTF-8");
    JValue root;
    try {
        root = json::Parser(h, n, kMaxDepth).document();
    } catch (const json::Error &e) {
        fail("the header is " + e.msg);
    }
    if (root.kind != JValue::OBJECT) fail("the header is not a JSON object");
    out.header_len = n;
    out.entries.clear();
    out.metadata.clear();
    std::vector<std::string> keys;
    keys.reserve(root.members.size());
    for (const auto &m : root.members) keys.push_back(m.first);
    std::sort(keys.begin(), keys.end());
    for (size_t i = 1; i < keys.size(); ++i)
        if (keys[i] == keys[i - 1]) fail("duplicate key '" + keys[i] + "'");
    for (const auto &m : root.members) {
        if (m.first == "__metadata__") {
            if (m.second.kind != JValue::OBJECT) fail("__metadata__ is not an object");
            std::vector<std::string> mk;
            for (const auto &kv : m.second.members) {
                if (std::find(mk.begin(), mk.end(), kv.first) != mk.end())
                    fail("duplicate metadata key '" + kv.first + "'");
                mk.push_back(kv.first);
                if (kv.second.kind != JValue::STRING) fail("metadata '" + kv.first + "' is not a string");
                out.metadata.emplace_back(kv.first, kv.second.text);
            }
        } else {
            out.entries.push_back(entry(data_len, m.first, m.second));
        }
    }
    // The tensors must tile the data section exactly.
    std::vector<const Entry *> by_offset;
    for (const auto &e : out.entries) by_offset.push_back(&e);
    std::sort(by_offset.begin(), by_offset.end(), [](const Entry *a, const Entry *b) {
        return a->begin != b->begin ? a->begin < b->begin : a->end < b->end;
    });
    uint64_t pos = 0;
    for (const Entry *e : by_offset) {
        if (e->begin < pos)
            fail(e->name + " overlaps the previous tensor (begins at " + std::to_string(e->begin) +
                 ", previous ends at " + std::to_string(pos) + ")");
        if (e->begin > pos)
            fail("hole before " + e->name + " (begins at " + std::to_string(e->begin) + ", previous ends at " +
                 std::to_string(pos) + ")");
        pos = e->end;
    }
    if (pos != data_len) fail(std::to_string(data_len - pos) + " bytes after the last tensor");
    std::sort(out.entries.begin(), out.entries.end(), [](const Entry &a, const Entry &b) { return a.name < b.name; });
    std::sort(out.metadata.begin(), out.metadata.end());
}

int dtype_size(int dtype) { return dtype >= 0 && dtype < 8 ? kDtypeSizes[dtype] : 0; }

}  // namespace st

struct StFile {
    std::string path;
    int fd = -1;
    const uint8_t *map = nullptr;
    uint64_t length = 0;
    st::Parsed parsed;
    std::unordered_map<std::string, size_t> index;
    ~StFile() {
        if (map && length) munmap((void *)map, length);
        if (fd >= 0) close(fd);
    }
};

}  // namespace lrm

using namespace lrm;

struct lrm_st_file_s {
    StFile f;
};

namespace {

lrm_status st_fail(lrm_status s, const std::string &m) {
    set_thread_error(m);
    return s;
}

void fill_entry(const lrm_st_file_s *h, const st::Entry &e, lrm_st_entry *out) {
    out->name = e.name.c_str();
    out->dtype = e.dtype;
    out->rank = (int32_t)e.shape.size();
    out->shape = e.shape.data();
    out->begin = e.begin;
    out->end = e.end;
    out->data = h->f.map + 8 + h->f.parsed.header_len + e.begin;
}

}  // namespace

extern "C" {

lrm_status lrm_st_validate(const void *bytes, uint64_t length, uint64_t *header_len, int64_t *count) {
    if (!bytes && length) return st_fail(LRM_ERR_ARGUMENT, "bytes is null");
    st::Parsed p;
    try {
        st::parse((const uint8_t *)bytes, length, p);
    } catch (const st::FormatError &e) {
        return st_fail(LRM_ERR_FORMAT, e.msg);
    } catch (const std::bad_alloc &) {
        return st_fail(LRM_ERR_OUT_OF_MEMORY, "out of host memory while parsing the header");
    }
    if (header_len) *header_len = p.header_len;
    if (count) *count = (int64_t)p.entries.size();
    return LRM_OK;
}

lrm_status lrm_st_open(const char *path, lrm_st_file *out) {
    if (!path || !out) return st_fail(LRM_ERR_ARGUMENT, "path or out is null");
    *out = nullptr;
    std::unique_ptr<lrm_st_file_s> h(new lrm_st_file_s);
    char real[4096];
    h->f.path = realpath(path, real) ? std::string(real) : std::string(path);
    h->f.fd = open(path, O_RDONLY | O_CLOEXEC);
    if (h->f.fd < 0) return st_fail(LRM_ERR_ARGUMENT, h->f.path + ": cannot open: " + strerror(errno));
    struct stat sb;
    if (fstat(h->f.fd, &sb) != 0) return st_fail(LRM_ERR_ARGUMENT, h->f.path + ": cannot stat: " + strerror(errno));
    h->f.length = (uint64_t)sb.st_size;
    if (h->f.length > 0) {
        void *m = mmap(nullptr, h->f.length, PROT_READ, MAP_PRIVATE, h->f.fd, 0);
        if (m == MAP_FAILED) return st_fail(LRM_ERR_ARGUMENT, h->f.path + ": cannot map: " + strerror(errno));
        h->f.map = (const uint8_t *)m;
    }
    try {
        st::parse(h->f.map, h->f.length, h->f.parsed);
    } catch (const st::FormatError &e) {
        return st_fail(LRM_ERR_FORMAT, h->f.path + ": " + e.msg);
    } catch (const std::bad_alloc &) {
        return st_fail(LRM_ERR_OUT_OF_MEMORY, h->f.path + ": out of host memory while parsing the header");
    }
    for (size_t i = 0; i < h->f.parsed.entries.size(); ++i) h->f.index[h->f.parsed.entries[i].name] = i;
    *out = h.release();
    return LRM_OK;
}

lrm_status lrm_st_close(lrm_st_file h) {
    delete h;
    return LRM_OK;
}

lrm_status lrm_st_info(lrm_st_file h, uint64_t *length, uint64_t *header_len, int64_t *count, int64_t *metadata_count,
                       int32_t *aligned) {
    if (!h) return st_fail(LRM_ERR_ARGUMENT, "file is null");
    const auto &p = h->f.parsed;
    if (length) *length = h->f.length;
    if (header_len) *header_len = p.header_len;
    if (count) *count = (int64_t)p.entries.size();
    if (metadata_count) *metadata_count = (int64_t)p.metadata.size();
    if (aligned) {
        bool ok = (8 + p.header_len) % 8 == 0;
        for (const auto &e : p.entries) ok = ok && e.begin % (uint64_t)st::dtype_size(e.dtype) == 0;
        *aligned = ok ? 1 : 0;
    }
    return LRM_OK;
}

lrm_status lrm_st_entry_at(lrm_st_file h, int64_t i, lrm_st_entry *out) {
    if (!h || !out) return st_fail(LRM_ERR_ARGUMENT, "file or out is null");
    if (i < 0 || i >= (int64_t)h->f.parsed.entries.size()) return st_fail(LRM_ERR_ARGUMENT, "entry index out of range");
    fill_entry(h, h->f.parsed.entries[(size_t)i], out);
    return LRM_OK;
}

lrm_status lrm_st_find(lrm_st_file h, const char *name, lrm_st_entry *out) {
    if (!h || !name || !out) return st_fail(LRM_ERR_ARGUMENT, "file, name or out is null");
    auto it = h->f.index.find(name);
    if (it == h->f.index.end()) return st_fail(LRM_ERR_ARGUMENT, h->f.path + ": no tensor '" + name + "'");
    fill_entry(h, h->f.parsed.entries[it->second], out);
    return LRM_OK;
}

lrm_status lrm_st_metadata_at(lrm_st_file h, int64_t i, const char **key, const char **value) {
    if (!h || !key || !value) return st_fail(LRM_ERR_ARGUMENT, "file, key or value is null");
    if (i < 0 || i >= (int64_t)h->f.parsed.metadata.size())
        return st_fail(LRM_ERR_ARGUMENT, "metadata index out of range");
    *key = h->f.parsed.metadata[(size_t)i].first.c_str();
    *value = h->f.parsed.metadata[(size_t)i].second.c_str();
    return LRM_OK;
}

}  // extern "C"
