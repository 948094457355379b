// dm_formats.cu — the reference's on-disk weight formats: the GGUF index with its block
// dequantisers, and the custom 4-bit quant file (256-byte JSON header + tensor records).
//
// Host side: index parsers that apply the reference's checks in the reference's order and
// with its messages (parse_gguf_index, reference src/format/gguf.mojo:257-411;
// scan_quant_file, reference src/format/quant_reader.mojo:520-662).  Device side: the
// GGUF block dequantisers (gguf.mojo:414-561, tools/oracle/oracle_port.py:68-159) and the
// two conversions into the HBM expert pool (asymmetric 4-bit, fp16 scale and uint4 zero
// per group): the exact one for the custom signed 4-bit format, and a round-to-nearest
// re-quantisation for everything else.  The ctx-level loaders that use these live in
// dm_api.cu.
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "dismoen_cuda.h"
#include "dm_internal.h"

// ------------------------------------------------------------------------------------
// shared host helpers
namespace {

void put_err(char* buf, uint64_t n, const char* type, const char* stage, const char* fmt, ...) {
    if (!buf || !n) return;
    char detail[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(detail, sizeof detail, fmt, ap);
    va_end(ap);
    for (char* p = detail; *p; ++p)
        if (*p == '"' || *p == '\\') *p = '\'';
    snprintf(buf, n, "{\"error_type\":\"%s\",\"detail\":\"%s\",\"stage\":\"%s\",\"layer\":-1}", type, detail, stage);
}

// Reads exactly n bytes at off; false on a short read or an error.
bool pread_all(int fd, void* dst, uint64_t n, uint64_t off) {
    auto* p = static_cast<uint8_t*>(dst);
    while (n) {
        const ssize_t r = pread(fd, p, n > (1u << 30) ? (1u << 30) : n, static_cast<off_t>(off));
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;
        p += r;
        off += static_cast<uint64_t>(r);
        n -= static_cast<uint64_t>(r);
    }
    return true;
}

bool mul_ok(uint64_t a, uint64_t b, uint64_t* out) {
    if (a && b > UINT64_MAX / a) return false;
    *out = a * b;
    return true;
}

// Little-endian reader over the header bytes (ByteReader, gguf.mojo:144-215): the same
// bounds, the same messages.
struct LeReader {
    const uint8_t* p;
    uint64_t n;
    uint64_t pos = 0;
    std::string err;
    bool fail(std::string m) {
        if (err.empty()) err = std::move(m);
        return false;
    }
    bool u8(uint64_t& v) {
        if (pos >= n) return fail("GGUF: unexpected EOF reading u8");
        v = p[pos++];
        return true;
    }
    bool u16(uint64_t& v) {
        if (pos + 2 > n) return fail("GGUF: unexpected EOF reading u16");
        v = static_cast<uint64_t>(p[pos]) | (static_cast<uint64_t>(p[pos + 1]) << 8);
        pos += 2;
        return true;
    }
    bool u32(uint64_t& v) {
        if (pos + 4 > n) return fail("GGUF: unexpected EOF reading u32");
        v = 0;
        for (int i = 0; i < 4; ++i) v |= static_cast<uint64_t>(p[pos + i]) << (8 * i);
        pos += 4;
        return true;
    }
    // read_u64 rejects values with the top bit set (the reference's Int is signed)
    bool u64(uint64_t& v) {
        if (pos + 8 > n) return fail("GGUF_FILE_CORRUPT: unexpected EOF reading u64");
        if (p[pos + 7] & 0x80) return fail("GGUF_FILE_CORRUPT: u64 overflow/negative value");
        v = 0;
        for (int i = 0; i < 8; ++i) v |= static_cast<uint64_t>(p[pos + i]) << (8 * i);
        pos += 8;
        return true;
    }
    bool str(std::string& s) {
        uint64_t len;
        if (!u64(len)) return false;
        if (len > 65536) return fail("GGUF: string length invalid: " + std::to_string(len));
        if (pos + len > n) return fail("GGUF: unexpected EOF reading string");
        s.assign(reinterpret_cast<const char*>(p + pos), len);
        pos += len;
        return true;
    }
};

// One metadata value as the string the reference stores in index.metadata
// (_skip_gguf_value, gguf.mojo:218-254): integers of 1/2/4/8 bytes (and f32/f64 as their
// raw bit patterns) in decimal, strings verbatim, arrays as "[Array of N elements]".
bool gguf_value(LeReader& r, uint64_t vtype, std::string& out, int depth) {
    uint64_t v = 0;
    switch (vtype) {
        case 0: case 1: case 7:
            if (!r.u8(v)) return false;
            out = std::to_string(v);
            return true;
        case 2: case 3:
            if (!r.u16(v)) return false;
            out = std::to_string(v);
            return true;
        case 4: case 5: case 6:
            if (!r.u32(v)) return false;
            out = std::to_string(v);
            return true;
        case 10: case 11: case 12:
            if (!r.u64(v)) return false;
            out = std::to_string(v);
            return true;
        case 8:
            return r.str(out);
        case 9: {
            uint64_t et, count;
            if (!r.u32(et) || !r.u64(count)) return false;
            if (depth > 16) return r.fail("GGUF_FILE_CORRUPT: metadata arrays nested too deeply");
            std::string tmp;
            for (uint64_t i = 0; i < count; ++i)
                if (!gguf_value(r, et, tmp, depth + 1)) return false;
            out = "[Array of " + std::to_string(count) + " elements]";
            return true;
        }
        default:
            return r.fail("GGUF: unknown value type " + std::to_string(vtype));
    }
}

// Int(String) of the reference: optional sign, decimal digits, nothing else.
bool parse_int(const std::string& s, long long* out) {
    size_t i = 0;
    bool neg = false;
    if (i < s.size() && (s[i] == '-' || s[i] == '+')) neg = s[i++] == '-';
    if (i == s.size()) return false;
    unsigned long long v = 0;
    for (; i < s.size(); ++i) {
        if (s[i] < '0' || s[i] > '9') return false;
        if (v > (ULLONG_MAX - 9) / 10) return false;
        v = v * 10 + static_cast<unsigned>(s[i] - '0');
    }
    if (v > static_cast<unsigned long long>(LLONG_MAX)) return false;
    *out = neg ? -static_cast<long long>(v) : static_cast<long long>(v);
    return true;
}

}  // namespace

// (block elements, bytes per block) of a GGML type (get_ggml_block_specs,
// gguf.mojo:76-102; unknown types fall back to (1, 4) there).
static void ggml_spec(int t, int* bs, int* bpb) {
    switch (t) {
        case DM_GGML_F32: *bs = 1; *bpb = 4; return;
        case DM_GGML_F16: case DM_GGML_BF16: *bs = 1; *bpb = 2; return;
        case 2: *bs = 32; *bpb = 18; return;   // Q4_0
        case 3: *bs = 32; *bpb = 20; return;   // Q4_1
        case DM_GGML_Q8_0: *bs = 32; *bpb = 34; return;
        case DM_GGML_Q3_K: *bs = 256; *bpb = 114; return;
        case DM_GGML_Q4_K: *bs = 256; *bpb = 144; return;
        case 13: *bs = 256; *bpb = 176; return;  // Q5_K
        case 14: *bs = 256; *bpb = 210; return;  // Q6_K
        case 18: *bs = 256; *bpb = 98; return;   // IQ3_XXS
        case 21: *bs = 256; *bpb = 110; return;  // IQ3_S
        default: *bs = 1; *bpb = 4; return;
    }
}

// ------------------------------------------------------------------------------------
// GGUF index
struct GgufTensor {
    std::string name;
    int ndim;
    uint64_t dims[8];
    int type;
    uint64_t offset, n_elements, raw_bytes;
};

struct dm_gguf {
    std::string path;
    int fd = -1;
    uint32_t version = 0;
    uint64_t tensor_count = 0, kv_count = 0, alignment = 32, data_offset = 0, file_size = 0;
    std::vector<GgufTensor> tensors;
    std::unordered_map<std::string, int64_t> map;
    std::vector<std::string> meta_keys;  // first-insertion order
    std::unordered_map<std::string, std::string> meta;
    ~dm_gguf() {
        if (fd >= 0) close(fd);
    }
};

extern "C" int32_t dm_ggml_block_spec(int32_t type, int32_t* block_elems, int32_t* block_bytes) {
    int bs, bpb;
    ggml_spec(type, &bs, &bpb);
    if (block_elems) *block_elems = bs;
    if (block_bytes) *block_bytes = bpb;
    return DM_OK;
}

extern "C" int32_t dm_gguf_open(const char* path, dm_gguf** out, char* err, uint64_t err_size) {
    if (!path || !out) {
        put_err(err, err_size, "WEIGHT_LOAD_FAILED", "gguf_index", "null argument");
        return DM_ERR_INVALID_ARG;
    }
    *out = nullptr;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
        put_err(err, err_size, "WEIGHT_LOAD_FAILED", "gguf_index", "cannot open %s: %s", path, strerror(errno));
        return DM_ERR_IO;
    }
    auto* g = new dm_gguf();
    g->path = path;
    g->fd = fd;
    auto corrupt = [&](const std::string& m) {
        put_err(err, err_size, "GGUF_FILE_CORRUPT", "gguf_index", "%s", m.c_str());
        delete g;
        return DM_ERR_FORMAT;
    };
    struct stat st;
    if (fstat(fd, &st) != 0) {
        put_err(err, err_size, "WEIGHT_LOAD_FAILED", "gguf_index", "cannot stat %s", path);
        delete g;
        return DM_ERR_IO;
    }
    const uint64_t filesize = static_cast<uint64_t>(st.st_size);
    g->file_size = filesize;
    if (filesize < 32)
        return corrupt("GGUF_FILE_CORRUPT: file size " + std::to_string(filesize) + " too small for header");
    // the header and tensor directory are read from the first 4 MiB, as in the reference
    const uint64_t head = filesize < (4ull << 20) ? filesize : (4ull << 20);
    std::vector<uint8_t> hb(head);
    if (!pread_all(fd, hb.data(), head, 0)) {
        put_err(err, err_size, "WEIGHT_LOAD_FAILED", "gguf_index", "short read of %s", path);
        delete g;
        return DM_ERR_IO;
    }
    LeReader r{hb.data(), head};
    uint64_t m0, m1, m2, m3;
    if (!r.u8(m0) || !r.u8(m1) || !r.u8(m2) || !r.u8(m3)) return corrupt(r.err);
    if (m0 != 0x47 || m1 != 0x47 || m2 != 0x55 || m3 != 0x46)
        return corrupt("GGUF_FILE_CORRUPT: invalid magic header (expected 'GGUF')");
    uint64_t v;
    if (!r.u32(v)) return corrupt(r.err);
    g->version = static_cast<uint32_t>(v);
    if (v != 2 && v != 3) return corrupt("GGUF_FILE_CORRUPT: unsupported version " + std::to_string(v));
    if (!r.u64(g->tensor_count) || !r.u64(g->kv_count)) return corrupt(r.err);
    if (g->tensor_count > 100000)
        return corrupt("GGUF_FILE_CORRUPT: tensor_count out of bounds: " + std::to_string(g->tensor_count));
    for (uint64_t k = 0; k < g->kv_count; ++k) {
        std::string key, val;
        uint64_t vt;
        if (!r.str(key) || !r.u32(vt) || !gguf_value(r, vt, val, 0)) return corrupt(r.err);
        if (!g->meta.count(key)) g->meta_keys.push_back(key);
        g->meta[key] = val;
        long long al;
        if (key == "general.alignment" && parse_int(val, &al) && al > 0) {
            if (al > (1ll << 30)) return corrupt("GGUF_FILE_CORRUPT: alignment out of range: " + val);
            g->alignment = static_cast<uint64_t>(al);
        }
    }
    uint64_t max_end = 0;
    g->tensors.reserve(g->tensor_count);
    for (uint64_t i = 0; i < g->tensor_count; ++i) {
        GgufTensor t{};
        uint64_t nd;
        if (!r.str(t.name) || !r.u32(nd)) return corrupt(r.err);
        if (nd < 1 || nd > 8) return corrupt("GGUF_FILE_CORRUPT: tensor ndim invalid: " + std::to_string(nd));
        t.ndim = static_cast<int>(nd);
        uint64_t ne = 1;
        for (int d = 0; d < t.ndim; ++d) {
            if (!r.u64(t.dims[d])) return corrupt(r.err);
            if (!mul_ok(ne, t.dims[d], &ne)) return corrupt("GGUF_FILE_CORRUPT: tensor element count overflow");
        }
        uint64_t ty;
        if (!r.u32(ty) || !r.u64(t.offset)) return corrupt(r.err);
        t.type = static_cast<int>(ty);
        t.n_elements = ne;
        int bs, bpb;
        ggml_spec(t.type, &bs, &bpb);
        const uint64_t nblocks = ne / bs + (ne % bs != 0);
        if (!mul_ok(nblocks, static_cast<uint64_t>(bpb), &t.raw_bytes))
            return corrupt("GGUF_FILE_CORRUPT: tensor offset integer overflow");
        const uint64_t end = t.offset + t.raw_bytes;
        if (end < t.offset || end > (1ull << 62)) return corrupt("GGUF_FILE_CORRUPT: tensor offset integer overflow");
        if (end > max_end) max_end = end;
        g->map[t.name] = static_cast<int64_t>(i);
        g->tensors.push_back(std::move(t));
    }
    const uint64_t al = g->alignment;
    const uint64_t data_start = (r.pos + al - 1) / al * al;
    g->data_offset = data_start;
    for (const GgufTensor& t : g->tensors)
        if (data_start + t.offset + t.raw_bytes > filesize)
            return corrupt("GGUF_FILE_CORRUPT: tensor extends beyond file boundary");
    // exact file size (the reference's F11b check): data start + end of the last tensor
    const uint64_t expected = data_start + max_end;
    if (filesize != expected) {
        const long long diff = static_cast<long long>(filesize) - static_cast<long long>(expected);
        return corrupt("GGUF_FILE_CORRUPT: actual size " + std::to_string(filesize) + " != expected size " +
                       std::to_string(expected) + " (diff: " + std::to_string(diff) + " bytes)");
    }
    *out = g;
    return DM_OK;
}

extern "C" void dm_gguf_close(dm_gguf* g) { delete g; }

extern "C" int32_t dm_gguf_summary(const dm_gguf* g, uint32_t* version, uint64_t* tensor_count,
                                   uint64_t* kv_count, uint64_t* alignment, uint64_t* data_offset,
                                   uint64_t* file_size) {
    if (!g) return DM_ERR_INVALID_ARG;
    if (version) *version = g->version;
    if (tensor_count) *tensor_count = g->tensor_count;
    if (kv_count) *kv_count = g->kv_count;
    if (alignment) *alignment = g->alignment;
    if (data_offset) *data_offset = g->data_offset;
    if (file_size) *file_size = g->file_size;
    return DM_OK;
}

extern "C" int32_t dm_gguf_tensor(const dm_gguf* g, int64_t i, dm_gguf_tensor_info* out) {
    if (!g || !out || i < 0 || i >= static_cast<int64_t>(g->tensors.size())) return DM_ERR_INVALID_ARG;
    const GgufTensor& t = g->tensors[i];
    memset(out, 0, sizeof *out);
    out->name = t.name.c_str();
    out->ndim = t.ndim;
    out->ggml_type = t.type;
    for (int d = 0; d < t.ndim; ++d) out->dims[d] = t.dims[d];
    out->offset = t.offset;
    out->file_offset = g->data_offset + t.offset;
    out->num_elements = t.n_elements;
    out->raw_bytes = t.raw_bytes;
    return DM_OK;
}

extern "C" int64_t dm_gguf_find(const dm_gguf* g, const char* name) {
    if (!g || !name) return -1;
    auto it = g->map.find(name);
    return it == g->map.end() ? -1 : it->second;
}

extern "C" int32_t dm_gguf_meta_key(const dm_gguf* g, int64_t i, char* buf, uint64_t size) {
    if (!g || !buf || !size || i < 0 || i >= static_cast<int64_t>(g->meta_keys.size())) return DM_ERR_INVALID_ARG;
    snprintf(buf, size, "%s", g->meta_keys[i].c_str());
    return g->meta_keys[i].size() < size ? DM_OK : DM_ERR_INVALID_ARG;
}

extern "C" int32_t dm_gguf_meta(const dm_gguf* g, const char* key, char* buf, uint64_t size) {
    if (!g || !key || !buf || !size) return DM_ERR_INVALID_ARG;
    auto it = g->meta.find(key);
    if (it == g->meta.end()) return DM_ERR_INVALID_ARG;
    snprintf(buf, size, "%s", it->second.c_str());
    return it->second.size() < size ? DM_OK : DM_ERR_INVALID_ARG;
}

extern "C" int32_t dm_gguf_read(const dm_gguf* g, int64_t i, uint64_t byte_offset, void* dst, uint64_t n) {
    if (!g || !dst || i < 0 || i >= static_cast<int64_t>(g->tensors.size())) return DM_ERR_INVALID_ARG;
    const GgufTensor& t = g->tensors[i];
    if (byte_offset > t.raw_bytes || n > t.raw_bytes - byte_offset) return DM_ERR_INVALID_ARG;
    return pread_all(g->fd, dst, n, g->data_offset + t.offset + byte_offset) ? DM_OK : DM_ERR_IO;
}

// ------------------------------------------------------------------------------------
// custom 4-bit quant file
namespace {

// JSON scanner for the header and the tensor records (the reference's Scanner): objects,
// strings with escapes, unsigned integers; other values are skipped.
struct Json {
    const char* s;
    size_t n, pos = 0;
    std::string err;
    bool fail(const std::string& m) {
        if (err.empty()) err = m;
        return false;
    }
    void ws() {
        while (pos < n && (s[pos] == ' ' || s[pos] == '\t' || s[pos] == '\n' || s[pos] == '\r')) ++pos;
    }
    int peek() {
        ws();
        return pos < n ? static_cast<unsigned char>(s[pos]) : -1;
    }
    bool expect(char c) {
        if (peek() != c) return fail(std::string("expected '") + c + "' at offset " + std::to_string(pos));
        ++pos;
        return true;
    }
    static void utf8(std::string& o, unsigned cp) {
        if (cp < 0x80) {
            o += static_cast<char>(cp);
        } else if (cp < 0x800) {
            o += static_cast<char>(0xC0 | (cp >> 6));
            o += static_cast<char>(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            o += static_cast<char>(0xE0 | (cp >> 12));
            o += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            o += static_cast<char>(0x80 | (cp & 0x3F));
        } else {
            o += static_cast<char>(0xF0 | (cp >> 18));
            o += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
            o += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            o += static_cast<char>(0x80 | (cp & 0x3F));
        }
    }
    bool hex4(unsigned* v) {
        if (pos + 4 > n) return fail("truncated \\u escape");
        *v = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = s[pos++];
            *v <<= 4;
            if (c >= '0' && c <= '9') *v |= c - '0';
            else if (c >= 'a' && c <= 'f') *v |= c - 'a' + 10;
            else if (c >= 'A' && c <= 'F') *v |= c - 'A' + 10;
            else return fail("bad \\u escape");
        }
        return true;
    }
    bool str(std::string& o) {
        if (!expect('"')) return false;
        o.clear();
        while (pos < n) {
            const char c = s[pos++];
            if (c == '"') return true;
            if (c != '\\') {
                o += c;
                continue;
            }
            if (pos >= n) break;
            const char e = s[pos++];
            switch (e) {
                case '"': o += '"'; break;
                case '\\': o += '\\'; break;
                case '/': o += '/'; break;
                case 'b': o += '\b'; break;
                case 'f': o += '\f'; break;
                case 'n': o += '\n'; break;
                case 'r': o += '\r'; break;
                case 't': o += '\t'; break;
                case 'u': {
                    unsigned cp;
                    if (!hex4(&cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00 && pos + 1 < n && s[pos] == '\\' && s[pos + 1] == 'u') {
                        pos += 2;
                        unsigned lo;
                        if (!hex4(&lo)) return false;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(o, cp);
                    break;
                }
                default: return fail("bad escape in string");
            }
        }
        return fail("unterminated string");
    }
    bool uint(uint64_t& v) {
        ws();
        if (pos >= n || s[pos] < '0' || s[pos] > '9') return fail("expected an unsigned integer at offset " + std::to_string(pos));
        v = 0;
        while (pos < n && s[pos] >= '0' && s[pos] <= '9') {
            if (v > (UINT64_MAX - 9) / 10) return fail("integer overflow");
            v = v * 10 + static_cast<unsigned>(s[pos++] - '0');
        }
        return true;
    }
    bool skip(int depth = 0) {
        if (depth > 32) return fail("JSON nested too deeply");
        const int c = peek();
        if (c == '"') {
            std::string t;
            return str(t);
        }
        if (c == '{' || c == '[') {
            const char close = c == '{' ? '}' : ']';
            ++pos;
            for (;;) {
                if (peek() == close) {
                    ++pos;
                    return true;
                }
                if (c == '{') {
                    std::string k;
                    if (!str(k) || !expect(':')) return false;
                }
                if (!skip(depth + 1)) return false;
                if (peek() == ',') ++pos;
                else if (peek() != close) return fail("expected ',' or a closing bracket");
            }
        }
        // number / true / false / null
        const size_t start = pos;
        while (pos < n && s[pos] != ',' && s[pos] != '}' && s[pos] != ']' && s[pos] != ' ' && s[pos] != '\n' &&
               s[pos] != '\t' && s[pos] != '\r')
            ++pos;
        return pos > start ? true : fail("expected a value");
    }
    // members of an object: fn(key) consumes the value
    template <class F>
    bool object(F&& fn) {
        if (!expect('{')) return false;
        for (;;) {
            if (peek() == '}') {
                ++pos;
                return true;
            }
            std::string key;
            if (!str(key) || !expect(':')) return false;
            if (!fn(key)) return false;
            if (peek() == ',') ++pos;
        }
    }
};

bool allowed_group(uint64_t g) { return g == 32 || g == 64 || g == 128 || g == 256; }

struct QTensor {
    std::string name, dtype, qdtype;
    std::vector<uint64_t> shape;
    uint64_t group, num_groups, scale_off, data_off;
    uint64_t n_elements, record_offset, payload_offset, scales_offset, data_offset, scales_bytes, weights_bytes;
};

}  // namespace

struct dm_quant_file {
    std::string path;
    int fd = -1;
    uint64_t version = 0, group_size = 0, num_tensors = 0, total_bytes = 0, file_size = 0;
    std::string model, format, scale_dtype;
    std::vector<QTensor> tensors;
    std::unordered_map<std::string, int64_t> map;
    ~dm_quant_file() {
        if (fd >= 0) close(fd);
    }
};

extern "C" int32_t dm_quant_file_open(const char* path, dm_quant_file** out, char* err, uint64_t err_size) {
    if (!path || !out) {
        put_err(err, err_size, "WEIGHT_LOAD_FAILED", "quant_index", "null argument");
        return DM_ERR_INVALID_ARG;
    }
    *out = nullptr;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
        put_err(err, err_size, "WEIGHT_LOAD_FAILED", "quant_index", "cannot open %s: %s", path, strerror(errno));
        return DM_ERR_IO;
    }
    auto* q = new dm_quant_file();
    q->path = path;
    q->fd = fd;
    auto bad = [&](const std::string& m) {
        put_err(err, err_size, "QUANT_FILE_CORRUPT", "quant_index", "%s", m.c_str());
        delete q;
        return DM_ERR_FORMAT;
    };
    struct stat st;
    if (fstat(fd, &st) != 0) {
        put_err(err, err_size, "WEIGHT_LOAD_FAILED", "quant_index", "cannot stat %s", path);
        delete q;
        return DM_ERR_IO;
    }
    const uint64_t fsz = static_cast<uint64_t>(st.st_size);
    q->file_size = fsz;
    constexpr uint64_t kHeader = 256;
    if (fsz < kHeader)
        return bad("scan_quant_file: file truncated, size " + std::to_string(fsz) + " < header size 256");
    char hdr[kHeader];
    if (!pread_all(fd, hdr, kHeader, 0)) return bad("scan_quant_file: short read of the header");
    // header (BlockHeader.from_bytes, quant_reader.mojo:96-168)
    {
        Json j{hdr, kHeader};
        q->version = 1;
        q->group_size = 64;
        q->scale_dtype = "FP16";
        const bool ok = j.object([&](const std::string& k) {
            if (k == "version") return j.uint(q->version);
            if (k == "model") return j.str(q->model);
            if (k == "num_tensors") return j.uint(q->num_tensors);
            if (k == "total_bytes") return j.uint(q->total_bytes);
            if (k == "quantization")
                return j.object([&](const std::string& qk) {
                    if (qk == "format") return j.str(q->format);
                    if (qk == "group_size") return j.uint(q->group_size);
                    if (qk == "scale_dtype") return j.str(q->scale_dtype);
                    return j.skip();
                });
            return j.skip();
        });
        if (!ok) return bad("scan_quant_file: failed parsing quant header: " + j.err);
    }
    // validate_block_header (quant_reader.mojo:344-383), in its order
    const std::string pre = "scan_quant_file: header validation failed (SEC-4): ";
    if (q->version != 1) return bad(pre + "Invalid quant header version: expected 1, got " + std::to_string(q->version));
    if (q->group_size == 0) return bad(pre + "Group size must be positive, got 0");
    if (!allowed_group(q->group_size))
        return bad(pre + "Group size must be one of {32, 64, 128, 256}, got " + std::to_string(q->group_size));
    if (q->format != "4-bit per-group") return bad(pre + "Unsupported quantization format: " + q->format);
    if (q->scale_dtype != "FP16") return bad(pre + "Unsupported scale dtype: " + q->scale_dtype);
    if (q->num_tensors == 0) return bad(pre + "Header num_tensors must be positive, got 0");
    if (q->num_tensors > 100000)
        return bad(pre + "Header num_tensors exceeds configured max: " + std::to_string(q->num_tensors) + " > 100000");
    if (q->total_bytes != fsz)
        return bad(pre + "File size mismatch: header total_bytes=" + std::to_string(q->total_bytes) +
                   ", physical size=" + std::to_string(fsz));
    uint64_t cur = kHeader;
    std::vector<char> js;
    for (uint64_t ti = 0; ti < q->num_tensors; ++ti) {
        if (cur + 4 > fsz)
            return bad("scan_quant_file: framing truncated before meta_len at tensor " + std::to_string(ti));
        uint8_t lb[4];
        if (!pread_all(fd, lb, 4, cur)) return bad("scan_quant_file: short read");
        const uint64_t mlen = lb[0] | (lb[1] << 8) | (lb[2] << 16) | (static_cast<uint64_t>(lb[3]) << 24);
        if (mlen == 0 || cur + 4 + mlen > fsz)
            return bad("scan_quant_file: invalid meta_len (" + std::to_string(mlen) + ") at offset " + std::to_string(cur));
        js.resize(mlen);
        if (!pread_all(fd, js.data(), mlen, cur + 4)) return bad("scan_quant_file: short read");
        QTensor t{};
        t.dtype = "BF16";
        t.qdtype = "4-bit";
        t.group = 64;
        const std::string mpre = "scan_quant_file: failed parsing tensor metadata JSON at tensor " + std::to_string(ti) + ": ";
        {
            Json j{js.data(), mlen};
            const bool ok = j.object([&](const std::string& k) {
                if (k == "name") return j.str(t.name);
                if (k == "dtype") return j.str(t.dtype);
                if (k == "quantized_dtype") return j.str(t.qdtype);
                if (k == "group_size") return j.uint(t.group);
                if (k == "num_groups") return j.uint(t.num_groups);
                if (k == "scale_offset") return j.uint(t.scale_off);
                if (k == "data_offset") return j.uint(t.data_off);
                if (k == "shape") {
                    if (!j.expect('[')) return false;
                    for (;;) {
                        if (j.peek() == ']') {
                            ++j.pos;
                            return true;
                        }
                        uint64_t d;
                        if (!j.uint(d)) return false;
                        t.shape.push_back(d);
                        if (j.peek() == ',') ++j.pos;
                    }
                }
                return j.skip();
            });
            if (!ok) return bad(mpre + j.err);
        }
        // the BlockTensorMeta constructor's own checks (quant_reader.mojo:183-206)
        if (!allowed_group(t.group)) return bad(mpre + "BlockTensorMeta: group_size not in {32, 64, 128, 256}");
        uint64_t ne = 1;
        bool ovf = false;
        for (uint64_t d : t.shape) ovf |= !mul_ok(ne, d, &ne);
        if (!ovf && ne % t.group != 0) return bad(mpre + "BlockTensorMeta: N % G != 0 (tail group not supported)");
        // validate_block_tensor_meta (quant_reader.mojo:385-433)
        const std::string vpre = "scan_quant_file: tensor metadata failed SEC-4 validation: ";
        if (t.name.empty()) return bad(vpre + "Tensor name cannot be empty");
        if (t.name.size() > 512)
            return bad(vpre + "Tensor name length exceeds configured max: " + std::to_string(t.name.size()) + " > 512");
        if (t.shape.empty()) return bad(vpre + "Tensor shape cannot be empty");
        if (t.shape.size() > 8)
            return bad(vpre + "Tensor ndim exceeds configured max: " + std::to_string(t.shape.size()) + " > 8");
        for (uint64_t d : t.shape)
            if (d == 0) return bad(vpre + "Dimension must be positive, got 0");
        if (ovf) return bad(vpre + "tensor element count overflow");
        if (t.num_groups != ne / t.group)
            return bad(vpre + "num_groups mismatch: meta=" + std::to_string(t.num_groups) +
                       ", expected=" + std::to_string(ne / t.group));
        t.n_elements = ne;
        t.scales_bytes = t.num_groups * 2;
        t.weights_bytes = (ne + 1) / 2;
        const uint64_t payload = t.scales_bytes + t.weights_bytes;
        const uint64_t rec = 4 + mlen + payload;
        if (cur + rec > fsz)
            return bad("scan_quant_file: tensor payload truncated: " + t.name + " (offset " +
                       std::to_string(cur + rec) + " > " + std::to_string(fsz) + ")");
        t.record_offset = cur;
        t.payload_offset = cur + 4 + mlen;
        t.scales_offset = t.payload_offset + t.scale_off;
        t.data_offset = t.payload_offset + t.data_off;
        // the scale and nibble ranges stay inside the record's payload (stricter than the
        // reference, which trusts the offsets)
        if (t.scale_off > payload || t.scales_bytes > payload - t.scale_off || t.data_off > payload ||
            t.weights_bytes > payload - t.data_off)
            return bad("scan_quant_file: scale/data offsets outside the payload of tensor " + t.name);
        q->map[t.name] = static_cast<int64_t>(q->tensors.size());
        q->tensors.push_back(std::move(t));
        cur += rec;
    }
    if (cur != fsz)
        return bad("scan_quant_file: trailing data or size mismatch (read " + std::to_string(cur) +
                   " != file_size " + std::to_string(fsz) + ")");
    *out = q;
    return DM_OK;
}

extern "C" void dm_quant_file_close(dm_quant_file* q) { delete q; }

extern "C" int32_t dm_quant_file_summary(const dm_quant_file* q, int32_t* version, int32_t* group_size,
                                         int64_t* num_tensors, uint64_t* total_bytes, char* model, uint64_t model_size) {
    if (!q) return DM_ERR_INVALID_ARG;
    if (version) *version = static_cast<int32_t>(q->version);
    if (group_size) *group_size = static_cast<int32_t>(q->group_size);
    if (num_tensors) *num_tensors = static_cast<int64_t>(q->tensors.size());
    if (total_bytes) *total_bytes = q->total_bytes;
    if (model && model_size) snprintf(model, model_size, "%s", q->model.c_str());
    return DM_OK;
}

extern "C" int32_t dm_quant_file_tensor(const dm_quant_file* q, int64_t i, dm_quant_tensor_info* out) {
    if (!q || !out || i < 0 || i >= static_cast<int64_t>(q->tensors.size())) return DM_ERR_INVALID_ARG;
    const QTensor& t = q->tensors[i];
    memset(out, 0, sizeof *out);
    out->name = t.name.c_str();
    out->dtype = t.dtype.c_str();
    out->ndim = static_cast<int32_t>(t.shape.size());
    for (size_t d = 0; d < t.shape.size(); ++d) out->shape[d] = t.shape[d];
    out->group_size = static_cast<int32_t>(t.group);
    out->num_groups = t.num_groups;
    out->num_elements = t.n_elements;
    out->record_offset = t.record_offset;
    out->scales_offset = t.scales_offset;
    out->data_offset = t.data_offset;
    out->scales_bytes = t.scales_bytes;
    out->weights_bytes = t.weights_bytes;
    return DM_OK;
}

extern "C" int64_t dm_quant_file_find(const dm_quant_file* q, const char* name) {
    if (!q || !name) return -1;
    auto it = q->map.find(name);
    return it == q->map.end() ? -1 : it->second;
}

extern "C" int32_t dm_quant_file_read(const dm_quant_file* q, int64_t i, int32_t part, uint64_t byte_offset,
                                      void* dst, uint64_t n) {
    if (!q || !dst || i < 0 || i >= static_cast<int64_t>(q->tensors.size()) || part < 0 || part > 1)
        return DM_ERR_INVALID_ARG;
    const QTensor& t = q->tensors[i];
    const uint64_t size = part == 0 ? t.scales_bytes : t.weights_bytes;
    const uint64_t base = part == 0 ? t.scales_offset : t.data_offset;
    if (byte_offset > size || n > size - byte_offset) return DM_ERR_INVALID_ARG;
    return pread_all(q->fd, dst, n, base + byte_offset) ? DM_OK : DM_ERR_IO;
}

// ------------------------------------------------------------------------------------
// device kernels
namespace dm {

static __device__ __forceinline__ float f16_at(const uint8_t* p) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(p[0] | (p[1] << 8))));
}

// Element e (0 <= e < block size) of one GGML block, as fp32 with the reference's
// rounding: every product and difference rounded separately (no contraction).
static __device__ __forceinline__ float gguf_elem(int type, const uint8_t* blk, int e, unsigned flags) {
    switch (type) {
        case DM_GGML_F32: {
            const uint32_t u = blk[0] | (blk[1] << 8) | (blk[2] << 16) | (static_cast<uint32_t>(blk[3]) << 24);
            return __uint_as_float(u);
        }
        case DM_GGML_F16: return f16_at(blk);
        case DM_GGML_BF16: return __uint_as_float(static_cast<uint32_t>(blk[0] | (blk[1] << 8)) << 16);
        case DM_GGML_Q8_0:  // gguf.mojo:414-441: fp16 scale, 32 int8
            return __fmul_rn(f16_at(blk), static_cast<float>(static_cast<int8_t>(blk[2 + e])));
        case DM_GGML_Q4_K: {  // gguf.mojo:444-506, oracle_port.py:86-127
            const float d = f16_at(blk), dmin = f16_at(blk + 2);
            const int j = e >> 5, i = e & 31;
            const uint8_t* sc = blk + 4;  // the 12 packed scale/min bytes
            int s6, m6;
            if (j < 4) {
                s6 = sc[j] & 63;
                m6 = sc[j + 4] & 63;
            } else if (flags & DM_GGUF_Q4K_MOJO) {  // gguf.mojo:478-485
                const int b4 = sc[j - 4], b8 = sc[j];
                s6 = (b8 & 0xF) | ((b4 >> 6) << 4);
                m6 = (b8 >> 4) | ((b8 >> 6) << 4);
            } else {  // the GGUF layout (oracle_port.py:108-112)
                s6 = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
                m6 = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
            }
            const uint8_t byte = blk[16 + j * 16 + (i & 15)];
            const int qv = i < 16 ? (byte & 0xF) : (byte >> 4);
            const float scv = __fmul_rn(static_cast<float>(s6), d);
            const float mv = __fmul_rn(static_cast<float>(m6), dmin);
            return __fsub_rn(__fmul_rn(scv, static_cast<float>(qv)), mv);
        }
        case DM_GGML_Q3_K: {  // gguf.mojo:509-560, oracle_port.py:130-159
            const float d = f16_at(blk + 112);
            const float scv = __fmul_rn(static_cast<float>(static_cast<int>(blk[96 + (e >> 4)]) - 32), d);
            const int h = (blk[e >> 3] >> (e & 7)) & 1;
            const int lo = (blk[32 + (e >> 2)] >> (2 * (e & 3))) & 3;
            return __fmul_rn(scv, static_cast<float>(((h << 2) | lo) - 4));
        }
        default: return 0.0f;
    }
}

__global__ void gguf_dequant_kernel(int type, int bs, int bpb, const uint8_t* __restrict__ raw, int64_t n,
                                    unsigned flags, float* __restrict__ out_f32, uint16_t* __restrict__ out_bf16) {
    for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < n;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = e / bs;
        const float v = gguf_elem(type, raw + b * bpb, static_cast<int>(e - b * bs), flags);
        if (out_f32) out_f32[e] = v;
        if (out_bf16) out_bf16[e] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    }
}

bool gguf_type_supported(int type) {
    return type == DM_GGML_F32 || type == DM_GGML_F16 || type == DM_GGML_BF16 || type == DM_GGML_Q8_0 ||
           type == DM_GGML_Q4_K || type == DM_GGML_Q3_K;
}

cudaError_t launch_gguf_dequant(cudaStream_t st, int type, const uint8_t* raw, int64_t n, unsigned flags,
                                float* out_f32, uint16_t* out_bf16) {
    int bs, bpb;
    ggml_spec(type, &bs, &bpb);
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    gguf_dequant_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(type, bs, bpb, raw, n, flags, out_f32, out_bf16);
    return cudaGetLastError();
}

// The custom signed 4-bit format (nibble n is n - 16 when n >= 8, else n; group scale s)
// into the pool's asymmetric form, exactly: q' = n XOR 8 is the nibble of q + 8 and
// w = s * q = s * (q' - 8), so zero = 8 and the scale carries over.  One thread per
// (row, pool group of gp elements) of the rows x cols slice starting at element e0 of the
// source tensor (e0, cols, gp even; gp | cols).  flags: bit 0 reserved nibble 0b1000,
// bit 1 a NaN / Inf / non-positive scale, bit 2 the source groups inside one pool group
// carry different scales (only possible when the source group is smaller than gp).
__global__ void sym4_to_pool_kernel(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales,
                                    int64_t e0, int rows, int cols, int gf, int gp, uint8_t* __restrict__ q_out,
                                    uint16_t* __restrict__ s_out, uint8_t* __restrict__ z_out, unsigned* flags) {
    const int ngp = cols / gp;
    const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (t >= static_cast<int64_t>(rows) * ngp) return;
    const int r = static_cast<int>(t / ngp), g = static_cast<int>(t % ngp);
    const int64_t base = e0 + static_cast<int64_t>(r) * cols + static_cast<int64_t>(g) * gp;
    unsigned f = 0;
    const uint8_t* src = packed + base / 2;
    uint8_t* dst = q_out + static_cast<int64_t>(r) * (cols / 2) + g * (gp / 2);
    for (int k = 0; k < gp / 2; ++k) {
        const uint8_t b = src[k];
        if ((b & 0xF) == 8 || (b >> 4) == 8) f |= 1u;
        dst[k] = b ^ 0x88;
    }
    const uint16_t s0 = scales[base / gf];
    for (int64_t e = base; e < base + gp; e += gf) {
        const uint16_t s = scales[e / gf];
        if (((s >> 10) & 0x1F) == 0x1F || (s & 0x8000u) || (s & 0x7FFFu) == 0) f |= 2u;
        if (s != s0) f |= 4u;
    }
    s_out[static_cast<int64_t>(r) * ngp + g] = s0;
    if ((g & 1) == 0) z_out[static_cast<int64_t>(r) * (ngp / 2) + g / 2] = 0x88;
    if (f) atomicOr(flags, f);
}

cudaError_t launch_sym4_to_pool(cudaStream_t st, const uint8_t* packed, const uint16_t* scales, int64_t e0, int rows,
                                int cols, int gf, int gp, uint8_t* q_out, uint16_t* s_out, uint8_t* z_out,
                                unsigned* flags) {
    const int64_t n = static_cast<int64_t>(rows) * (cols / gp);
    sym4_to_pool_kernel<<<static_cast<unsigned>((n + 127) / 128), 128, 0, st>>>(packed, scales, e0, rows, cols, gf, gp,
                                                                              q_out, s_out, z_out, flags);
    return cudaGetLastError();
}

// Round-to-nearest re-quantisation of fp32 weights [rows][cols] into the pool's form, per
// group of gp along the row: lo = min(0, min w), hi = max(0, max w);
// s = fp16(RN((hi - lo) / 15)) (saturated to [2^-24, 65504]; 1 when hi == lo);
// z = clamp(rint(-lo / s), 0, 15); q = clamp(rint(w / s) + z, 0, 15); every division and
// rint rounds to nearest even.  One thread per (row, pair of groups) so that the zero
// byte (two groups) has one writer.  flags bit 3: a non-finite weight.  *max_err_bits
// receives the largest |w - s (q - z)| (fp32 bits, atomic max).
__global__ void requant_pool_kernel(const float* __restrict__ w, int rows, int cols, int gp,
                                    uint8_t* __restrict__ q_out, uint16_t* __restrict__ s_out,
                                    uint8_t* __restrict__ z_out, unsigned* flags, unsigned* max_err_bits) {
    const int npair = cols / (2 * gp);
    const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (t >= static_cast<int64_t>(rows) * npair) return;
    const int r = static_cast<int>(t / npair), pr = static_cast<int>(t % npair);
    float err = 0.0f;
    unsigned f = 0;
    uint8_t zb = 0;
    for (int h = 0; h < 2; ++h) {
        const int g = 2 * pr + h;
        const float* src = w + static_cast<int64_t>(r) * cols + static_cast<int64_t>(g) * gp;
        float lo = 0.0f, hi = 0.0f;
        for (int k = 0; k < gp; ++k) {
            const float v = src[k];
            if (!isfinite(v)) f |= 8u;
            lo = fminf(lo, v);
            hi = fmaxf(hi, v);
        }
        float s32 = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
        uint16_t s16;
        if (s32 == 0.0f || !isfinite(s32)) {
            s16 = isfinite(s32) ? 0x3C00 : 0x7BFF;
        } else {
            s16 = __half_as_ushort(__float2half_rn(s32));
            if ((s16 & 0x7FFF) == 0x7C00) s16 = 0x7BFF;
            if (s16 == 0) s16 = 0x0001;
        }
        const float s = __half2float(__ushort_as_half(s16));
        const float zf = fminf(fmaxf(rintf(__fdiv_rn(-lo, s)), 0.0f), 15.0f);
        const int z = static_cast<int>(zf);
        uint8_t* dst = q_out + static_cast<int64_t>(r) * (cols / 2) + g * (gp / 2);
        for (int k = 0; k < gp; k += 2) {
            int qq[2];
            for (int u = 0; u < 2; ++u) {
                const float v = src[k + u];
                const float qf = fminf(fmaxf(__fadd_rn(rintf(__fdiv_rn(v, s)), zf), 0.0f), 15.0f);
                qq[u] = isfinite(v) ? static_cast<int>(qf) : z;
                const float rec = __fmul_rn(s, static_cast<float>(qq[u] - z));
                const float d = fabsf(__fsub_rn(v, rec));
                if (isfinite(v)) err = fmaxf(err, d);
            }
            dst[k / 2] = static_cast<uint8_t>(qq[0] | (qq[1] << 4));
        }
        s_out[static_cast<int64_t>(r) * (cols / gp) + g] = s16;
        zb |= static_cast<uint8_t>(z << (4 * h));
    }
    z_out[static_cast<int64_t>(r) * npair + pr] = zb;
    if (f) atomicOr(flags, f);
    atomicMax(max_err_bits, __float_as_uint(err));
}

cudaError_t launch_requant_pool(cudaStream_t st, const float* w, int rows, int cols, int gp, uint8_t* q_out,
                                uint16_t* s_out, uint8_t* z_out, unsigned* flags, unsigned* max_err_bits) {
    const int64_t n = static_cast<int64_t>(rows) * (cols / (2 * gp));
    requant_pool_kernel<<<static_cast<unsigned>((n + 127) / 128), 128, 0, st>>>(w, rows, cols, gp, q_out, s_out,
                                                                              z_out, flags, max_err_bits);
    return cudaGetLastError();
}

}  // namespace dm
