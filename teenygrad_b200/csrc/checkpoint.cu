// Checkpoint ingest: safetensors files, including teeny-quant's int8 output.
//
// A .safetensors file is an 8-byte little-endian header length, a JSON header
// {"name": {"dtype", "shape", "data_offsets": [begin, end]}, ...,
// "__metadata__": {string: string}} and the tensor bytes (offsets relative to
// the end of the header).  The file is memory-mapped and read in place, as the
// reference's loader does (utilities/teeny-data/src/safetensors/mod.rs:22-45).
//
// teeny-quant writes its quantised checkpoints in the compressed-tensors
// convention (utilities/teeny-quant/src/format.rs:17-35, quantize_tensor
// :145-182): a quantised `foo.weight` holds I8 values of the original shape,
// `foo.weight_scale` one F32 scale per output channel, and the header's
// `quantization_config` metadata describes the scheme.  Those tensors are
// copied as they are into the decoder's int8 GEMV layout (no re-quantisation).
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <map>
#include <string>
#include <vector>

#include "tb_internal.h"

struct tb_st {
    struct Tensor {
        int dtype = -1;              // TB_F32 / TB_BF16 / TB_I8 / TB_I32, or -1 (other)
        std::string dtype_name;
        std::vector<int64_t> shape;
        const uint8_t* data = nullptr;
        size_t bytes = 0;
    };
    void* map = nullptr;
    size_t map_bytes = 0;
    std::map<std::string, Tensor> tensors;
    std::map<std::string, std::string> metadata;
    std::vector<std::string> names;   // header order
    std::string error;
};

namespace {

// Minimal JSON reader for the safetensors header (objects, arrays, strings,
// numbers, literals).
struct Json {
    const char* p;
    const char* end;
    std::string err;

    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    bool expect(char c) {
        ws();
        if (p < end && *p == c) {
            p++;
            return true;
        }
        err = std::string("expected '") + c + "'";
        return false;
    }
    bool string(std::string& out) {
        ws();
        if (p >= end || *p != '"') {
            err = "expected a string";
            return false;
        }
        p++;
        out.clear();
        while (p < end && *p != '"') {
            char c = *p++;
            if (c == '\\') {
                if (p >= end) break;
                char e = *p++;
                switch (e) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {
                        if (end - p < 4) {
                            err = "bad \\u escape";
                            return false;
                        }
                        unsigned v = 0;
                        for (int i = 0; i < 4; i++) {
                            char h = *p++;
                            v = v * 16 + (unsigned)(h >= '0' && h <= '9' ? h - '0' : (h | 32) - 'a' + 10);
                        }
                        if (v < 0x80) {
                            out += (char)v;
                        } else if (v < 0x800) {
                            out += (char)(0xC0 | (v >> 6));
                            out += (char)(0x80 | (v & 63));
                        } else {
                            out += (char)(0xE0 | (v >> 12));
                            out += (char)(0x80 | ((v >> 6) & 63));
                            out += (char)(0x80 | (v & 63));
                        }
                        break;
                    }
                    default: out += e;
                }
            } else {
                out += c;
            }
        }
        if (p >= end) {
            err = "unterminated string";
            return false;
        }
        p++;
        return true;
    }
    bool integer(int64_t& v) {
        ws();
        bool neg = false;
        if (p < end && *p == '-') {
            neg = true;
            p++;
        }
        if (p >= end || *p < '0' || *p > '9') {
            err = "expected an integer";
            return false;
        }
        v = 0;
        while (p < end && *p >= '0' && *p <= '9') v = v * 10 + (*p++ - '0');
        if (neg) v = -v;
        return true;
    }
    // Skips any value (used for unknown keys).
    bool skip() {
        ws();
        if (p >= end) return false;
        if (*p == '"') {
            std::string s;
            return string(s);
        }
        if (*p == '{' || *p == '[') {
            const char close = *p == '{' ? '}' : ']';
            const bool obj = *p == '{';
            p++;
            ws();
            if (p < end && *p == close) {
                p++;
                return true;
            }
            while (true) {
                if (obj) {
                    std::string k;
                    if (!string(k) || !expect(':')) return false;
                }
                if (!skip()) return false;
                ws();
                if (p < end && *p == ',') {
                    p++;
                    continue;
                }
                return expect(close);
            }
        }
        while (p < end && *p != ',' && *p != '}' && *p != ']') p++;   // number / literal
        return true;
    }
};

int dtype_of(const std::string& s) {
    if (s == "F32") return TB_F32;
    if (s == "BF16") return TB_BF16;
    if (s == "I8") return TB_I8;
    if (s == "I32") return TB_I32;
    return -1;
}

size_t dtype_bytes(const std::string& s) {
    if (s == "F64" || s == "I64" || s == "U64") return 8;
    if (s == "F32" || s == "I32" || s == "U32") return 4;
    if (s == "F16" || s == "BF16" || s == "I16" || s == "U16") return 2;
    return 1;   // I8, U8, BOOL, F8_*
}

bool parse_header(tb_st* st, const char* h, size_t n, const uint8_t* data, size_t data_bytes) {
    Json j{h, h + n, {}};
    if (!j.expect('{')) return st->error = j.err, false;
    j.ws();
    if (j.p < j.end && *j.p == '}') return true;
    while (true) {
        std::string name;
        if (!j.string(name) || !j.expect(':')) return st->error = "header: " + j.err, false;
        if (name == "__metadata__") {
            if (!j.expect('{')) return st->error = "header: " + j.err, false;
            j.ws();
            if (j.p < j.end && *j.p == '}') {
                j.p++;
            } else {
                while (true) {
                    std::string k, v;
                    if (!j.string(k) || !j.expect(':') || !j.string(v)) return st->error = "metadata: " + j.err, false;
                    st->metadata[k] = v;
                    j.ws();
                    if (j.p < j.end && *j.p == ',') {
                        j.p++;
                        continue;
                    }
                    if (!j.expect('}')) return st->error = "metadata: " + j.err, false;
                    break;
                }
            }
        } else {
            tb_st::Tensor t;
            int64_t b0 = -1, b1 = -1;
            if (!j.expect('{')) return st->error = "tensor " + name + ": " + j.err, false;
            while (true) {
                std::string k;
                if (!j.string(k) || !j.expect(':')) return st->error = "tensor " + name + ": " + j.err, false;
                if (k == "dtype") {
                    if (!j.string(t.dtype_name)) return st->error = "tensor " + name + ": " + j.err, false;
                    t.dtype = dtype_of(t.dtype_name);
                } else if (k == "shape") {
                    if (!j.expect('[')) return st->error = "tensor " + name + ": " + j.err, false;
                    j.ws();
                    if (j.p < j.end && *j.p == ']') {
                        j.p++;
                    } else {
                        while (true) {
                            int64_t v;
                            if (!j.integer(v)) return st->error = "tensor " + name + ": " + j.err, false;
                            t.shape.push_back(v);
                            j.ws();
                            if (j.p < j.end && *j.p == ',') {
                                j.p++;
                                continue;
                            }
                            if (!j.expect(']')) return st->error = "tensor " + name + ": " + j.err, false;
                            break;
                        }
                    }
                } else if (k == "data_offsets") {
                    if (!j.expect('[') || !j.integer(b0) || !j.expect(',') || !j.integer(b1) || !j.expect(']'))
                        return st->error = "tensor " + name + ": " + j.err, false;
                } else if (!j.skip()) {
                    return st->error = "tensor " + name + ": bad value", false;
                }
                j.ws();
                if (j.p < j.end && *j.p == ',') {
                    j.p++;
                    continue;
                }
                if (!j.expect('}')) return st->error = "tensor " + name + ": " + j.err, false;
                break;
            }
            size_t elems = 1;
            for (int64_t d : t.shape) {
                if (d < 0) return st->error = "tensor " + name + ": negative dimension", false;
                elems *= (size_t)d;
            }
            if (b0 < 0 || b1 < b0 || (size_t)b1 > data_bytes)
                return st->error = "tensor " + name + ": data_offsets outside the file", false;
            if ((size_t)(b1 - b0) != elems * dtype_bytes(t.dtype_name) && t.dtype >= 0)
                return st->error = "tensor " + name + ": byte size does not match shape and dtype", false;
            t.data = data + b0;
            t.bytes = (size_t)(b1 - b0);
            st->names.push_back(name);
            st->tensors[name] = t;
        }
        j.ws();
        if (j.p < j.end && *j.p == ',') {
            j.p++;
            continue;
        }
        if (!j.expect('}')) return st->error = "header: " + j.err, false;
        return true;
    }
}

}  // namespace

extern "C" {

int tb_st_open(const char* path, tb_st** out) {
    if (!path || !out) return TB_ERR_ARG;
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return TB_ERR_ARG;
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
        close(fd);
        return TB_ERR_SHAPE;
    }
    void* m = mmap(nullptr, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return TB_ERR_ARG;
    tb_st* st = new tb_st();
    st->map = m;
    st->map_bytes = (size_t)sb.st_size;
    const uint8_t* b = reinterpret_cast<const uint8_t*>(m);
    uint64_t hn = 0;
    for (int i = 0; i < 8; i++) hn |= (uint64_t)b[i] << (8 * i);
    if (hn > st->map_bytes - 8 ||
        !parse_header(st, reinterpret_cast<const char*>(b + 8), (size_t)hn, b + 8 + hn, st->map_bytes - 8 - hn)) {
        if (st->error.empty()) st->error = "header length outside the file";
        fprintf(stderr, "tb_st_open(%s): %s\n", path, st->error.c_str());
        munmap(st->map, st->map_bytes);
        delete st;
        return TB_ERR_SHAPE;
    }
    *out = st;
    return TB_OK;
}

int tb_st_close(tb_st* st) {
    if (!st) return TB_OK;
    if (st->map) munmap(st->map, st->map_bytes);
    delete st;
    return TB_OK;
}

int tb_st_count(tb_st* st) { return st ? (int)st->names.size() : -1; }

const char* tb_st_name(tb_st* st, int i) {
    if (!st || i < 0 || i >= (int)st->names.size()) return nullptr;
    return st->names[i].c_str();
}

int tb_st_tensor(tb_st* st, const char* name, int* dtype, int64_t* shape, int* rank, const void** data,
                 size_t* bytes) {
    if (!st || !name) return TB_ERR_ARG;
    auto it = st->tensors.find(name);
    if (it == st->tensors.end()) return TB_ERR_ARG;
    const tb_st::Tensor& t = it->second;
    if (dtype) *dtype = t.dtype;
    if (rank) {
        const int r = (int)t.shape.size();
        if (shape && r > *rank) return TB_ERR_SHAPE;
        if (shape)
            for (int i = 0; i < r; i++) shape[i] = t.shape[i];
        *rank = r;
    }
    if (data) *data = t.data;
    if (bytes) *bytes = t.bytes;
    return TB_OK;
}

const char* tb_st_metadata(tb_st* st, const char* key) {
    if (!st || !key) return nullptr;
    auto it = st->metadata.find(key);
    return it == st->metadata.end() ? nullptr : it->second.c_str();
}

}  // extern "C"
