// gguf.cpp -- GGUF v2/v3 reader: the host-side mirror of src/reader.rs and
// the parsing half of src/lib.rs:29-138 load_model.  Every read is bounds
// checked (src/reader.rs:25-37 `take`); a truncated or lying file becomes a
// status code with the reference's error message, never a crash.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <string>

#include "host.h"

tir_gguf::~tir_gguf() {
    if (map_base) munmap(map_base, map_len);
}

namespace tir {

namespace {

struct ReadErr {
    tir_status st;
    std::string msg;
};

// src/error.rs:5-24 Display strings.
ReadErr eof(const char* what, size_t off) {
    return {TIR_ERR_UNEXPECTED_EOF,
            std::string("unexpected end of file reading ") + what + " at offset " + std::to_string(off)};
}

class Reader {
   public:
    Reader(const uint8_t* d, size_t n) : d_(d), n_(n) {}

    // src/reader.rs:25-37
    bool take(size_t off, size_t len, const char* what, const uint8_t*& out, ReadErr& e) const {
        size_t end;
        if (__builtin_add_overflow(off, len, &end) || end > n_ || off > n_) {
            e = eof(what, off);
            return false;
        }
        out = d_ + off;
        return true;
    }
    bool u32(size_t& off, const char* what, uint32_t& v, ReadErr& e) const {
        const uint8_t* p;
        if (!take(off, 4, what, p, e)) return false;
        std::memcpy(&v, p, 4);
        off += 4;
        return true;
    }
    bool u64(size_t& off, const char* what, uint64_t& v, ReadErr& e) const {
        const uint8_t* p;
        if (!take(off, 8, what, p, e)) return false;
        std::memcpy(&v, p, 8);
        off += 8;
        return true;
    }

   private:
    const uint8_t* d_;
    size_t n_;
};

// Rust str::from_utf8 acceptance (RFC 3629: no overlongs, no surrogates,
// nothing above U+10FFFF).
bool valid_utf8(const uint8_t* s, size_t n) {
    size_t i = 0;
    while (i < n) {
        const uint8_t c = s[i];
        if (c < 0x80) {
            ++i;
            continue;
        }
        size_t len;
        uint32_t cp;
        if ((c & 0xE0) == 0xC0) {
            len = 2;
            cp = c & 0x1F;
        } else if ((c & 0xF0) == 0xE0) {
            len = 3;
            cp = c & 0x0F;
        } else if ((c & 0xF8) == 0xF0) {
            len = 4;
            cp = c & 0x07;
        } else {
            return false;
        }
        if (i + len > n) return false;
        for (size_t j = 1; j < len; ++j) {
            if ((s[i + j] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (s[i + j] & 0x3F);
        }
        if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000)) return false;
        if (cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
        i += len;
    }
    return true;
}

// src/reader.rs:191-199 parse_string
bool parse_string(const Reader& r, size_t& off, std::string& out, ReadErr& e) {
    uint64_t n;
    if (!r.u64(off, "string length", n, e)) return false;
    const uint8_t* p;
    if (n > SIZE_MAX || !r.take(off, static_cast<size_t>(n), "string bytes", p, e)) {
        if (n > SIZE_MAX) e = eof("string bytes", off);
        return false;
    }
    if (!valid_utf8(p, static_cast<size_t>(n))) {
        e = {TIR_ERR_INVALID_UTF8, "invalid utf8 in string at offset " + std::to_string(off)};
        return false;
    }
    out.assign(reinterpret_cast<const char*>(p), static_cast<size_t>(n));
    off += static_cast<size_t>(n);
    return true;
}

// src/reader.rs:50-96 read_scalar (widths: src/reader.rs:89-96)
bool read_scalar(const Reader& r, size_t& off, uint32_t vtype, MetaValue& v, ReadErr& e) {
    static const char* names[] = {"u8", "i8", "u16", "i16", "u32", "i32", "f32", "bool", "", "", "u64", "i64", "f64"};
    size_t width;
    switch (vtype) {
        case 0: case 1: case 7: width = 1; break;
        case 2: case 3: width = 2; break;
        case 4: case 5: case 6: width = 4; break;
        case 10: case 11: case 12: width = 8; break;
        default:
            e = {TIR_ERR_UNSUPPORTED_TYPE, "unsupported metadata value type: " + std::to_string(vtype)};
            return false;
    }
    const uint8_t* p;
    if (!r.take(off, width, names[vtype], p, e)) return false;
    v.vtype = vtype;
    switch (vtype) {
        case 0: v.u = p[0]; break;
        case 1: v.i = static_cast<int8_t>(p[0]); break;
        case 2: { uint16_t x; std::memcpy(&x, p, 2); v.u = x; break; }
        case 3: { int16_t x; std::memcpy(&x, p, 2); v.i = x; break; }
        case 4: { uint32_t x; std::memcpy(&x, p, 4); v.u = x; break; }
        case 5: { int32_t x; std::memcpy(&x, p, 4); v.i = x; break; }
        case 6: { float x; std::memcpy(&x, p, 4); v.f = x; break; }
        case 7: v.u = p[0] != 0; break;
        case 10: { uint64_t x; std::memcpy(&x, p, 8); v.u = x; break; }
        case 11: { int64_t x; std::memcpy(&x, p, 8); v.i = x; break; }
        case 12: { double x; std::memcpy(&x, p, 8); v.f = x; break; }
    }
    off += width;
    return true;
}

bool parse_general_impl(const Reader& r, size_t& off, uint64_t count, std::vector<MetaField>& out,
                        ReadErr& e) {
    while (count != 0) {
        MetaField fld;
        if (!parse_string(r, off, fld.name, e)) return false;
        uint32_t ftype;
        if (!r.u32(off, "field type", ftype, e)) return false;
        if (ftype == TIR_GGUF_STRING) {
            fld.value.vtype = TIR_GGUF_STRING;
            if (!parse_string(r, off, fld.value.str, e)) return false;
        } else if (ftype == TIR_GGUF_ARRAY) {
            uint32_t et;
            uint64_t n;
            if (!r.u32(off, "array element type", et, e)) return false;
            if (!r.u64(off, "array length", n, e)) return false;
            fld.value.vtype = TIR_GGUF_ARRAY;
            fld.value.array_type = et;
            for (uint64_t j = 0; j < n; ++j) {
                MetaValue item;
                if (et == TIR_GGUF_STRING) {
                    item.vtype = TIR_GGUF_STRING;
                    if (!parse_string(r, off, item.str, e)) return false;
                } else if (!read_scalar(r, off, et, item, e)) {  // nested arrays -> UnsupportedType(9)
                    return false;
                }
                fld.value.items.push_back(std::move(item));
            }
        } else if (!read_scalar(r, off, ftype, fld.value, e)) {
            return false;
        }
        out.push_back(std::move(fld));
        --count;
    }
    return true;
}

}  // namespace

tir_status gguf_parse_general(const uint8_t* map, size_t len, size_t offset, uint64_t count,
                              std::vector<MetaField>& out, size_t& end) {
    Reader r(map, len);
    ReadErr e;
    size_t off = offset;
    if (!parse_general_impl(r, off, count, out, e)) return fail(e.st, e.msg);
    end = off;
    return TIR_OK;
}

const TensorInfo* gguf_find(const tir_gguf* g, const std::string& name) {
    auto it = g->index.find(name);
    return it == g->index.end() ? nullptr : &g->tensors[it->second];
}

// src/lib.rs:29-138 load_model (parse only).
tir_status gguf_parse_all(tir_gguf* g) {
    const uint8_t* map = g->data;
    const size_t len = g->len;
    Reader r(map, len);
    ReadErr e;
    auto reader_fail = [](const ReadErr& er) { return fail(er.st, "Reader Error: " + er.msg); };
    if (len < 24) return reader_fail(eof("gguf header", len));
    if (std::memcmp(map, "GGUF", 4) != 0) return reader_fail({TIR_ERR_BAD_MAGIC, "bad magic number, not a gguf file"});
    uint32_t version;
    std::memcpy(&version, map + 4, 4);
    if (version < 2 || version > 3)
        return reader_fail({TIR_ERR_BAD_VERSION, "unsupported gguf version: " + std::to_string(version)});
    g->version = version;
    uint64_t n_tensors, n_kv;
    std::memcpy(&n_tensors, map + 8, 8);
    std::memcpy(&n_kv, map + 16, 8);
    size_t off = 24;
    if (!parse_general_impl(r, off, n_kv, g->fields, e)) return reader_fail(e);

    // src/lib.rs:70-97: each key only counts with its exact wire type.
    bool have[6] = {false, false, false, false, false, false};
    tir_transformer t{};
    uint64_t alignment = 32;
    for (const MetaField& f : g->fields) {
        const MetaValue& v = f.value;
        if (f.name == "llama.block_count" && v.vtype == TIR_GGUF_U32) { t.layers = static_cast<uint32_t>(v.u); have[0] = true; }
        else if (f.name == "llama.rope.dimension_count" && v.vtype == TIR_GGUF_U32) { t.dim = v.u; have[1] = true; }
        else if (f.name == "llama.embedding_length" && v.vtype == TIR_GGUF_U32) { t.embed_dim = v.u; have[2] = true; }
        else if (f.name == "llama.attention.head_count" && v.vtype == TIR_GGUF_U32) { t.q_heads = v.u; have[3] = true; }
        else if (f.name == "llama.attention.head_count_kv" && v.vtype == TIR_GGUF_U32) { t.k_v_heads = v.u; have[4] = true; }
        else if (f.name == "llama.rope.freq_base" && v.vtype == TIR_GGUF_F32) { t.base_freq = static_cast<float>(v.f); have[5] = true; }
        else if (f.name == "general.alignment" && v.vtype == TIR_GGUF_U32) { alignment = v.u; }
    }
    static const char* labels[6] = {"Layers", "Dimension", "Embedding Length", "Query Attention Heads",
                                    "K/V Attention Heads", "Rope Base Frequency"};
    for (int i = 0; i < 6; ++i)
        if (!have[i])
            return fail(TIR_ERR_MISSING_FIELD, std::string("Metadata Load error: missing required field: ") + labels[i]);
    if (alignment == 0) return reader_fail({TIR_ERR_UNEXPECTED_EOF, "unexpected end of file reading alignment at offset 0"});

    // src/reader.rs:201-238 parse_tensors
    for (uint64_t ti = 0; ti < n_tensors; ++ti) {
        TensorInfo info;
        if (!parse_string(r, off, info.name, e)) return reader_fail(e);
        if (!r.u32(off, "tensor dimension count", info.n_dims, e)) return reader_fail(e);
        for (uint32_t di = 0; di < info.n_dims; ++di) {
            uint64_t v;
            if (!r.u64(off, "tensor dimension", v, e)) return reader_fail(e);
            info.shape.push_back(v);
        }
        if (!r.u32(off, "tensor dtype", info.dtype, e)) return reader_fail(e);
        const uint8_t* p;
        if (!r.take(off, 8, "tensor offset", p, e)) return reader_fail(e);
        std::memcpy(&info.offset, p, 8);
        off += 8;
        g->tensors.push_back(std::move(info));
    }
    // src/lib.rs:120-122: data starts at the next aligned boundary.
    const size_t data_start = (off + alignment - 1) / alignment * alignment;

    // src/reader.rs:240-283 parse_tensor_data / parse_q8 / parse_f32
    for (size_t ti = 0; ti < g->tensors.size(); ++ti) {
        TensorInfo& info = g->tensors[ti];
        uint64_t count = 1;
        bool overflow = false;
        for (uint64_t s : info.shape) overflow |= __builtin_mul_overflow(count, s, &count);
        ReadErr te;
        const uint8_t* pd = nullptr;
        bool ok = true;
        size_t bytes = 0;
        const size_t toff = data_start + static_cast<size_t>(info.offset);
        if (info.dtype == TIR_DTYPE_F32) {
            overflow |= __builtin_mul_overflow(count, 4ull, &count);
            bytes = static_cast<size_t>(count);
            if (overflow) { te = eof("f32 tensor data", toff); ok = false; }
            else ok = r.take(toff, bytes, "f32 tensor data", pd, te);
        } else if (info.dtype == TIR_DTYPE_Q8_0) {
            if (count % 32 != 0) {
                te = {TIR_ERR_BAD_QUANT_BLOCK, "q8_0 tensor length " + std::to_string(count) + " is not a multiple of 32"};
                ok = false;
            } else {
                bytes = static_cast<size_t>(count / 32 * 34);
                if (overflow) { te = eof("q8_0 tensor data", toff); ok = false; }
                else ok = r.take(toff, bytes, "q8_0 tensor data", pd, te);
            }
        } else {
            te = {TIR_ERR_UNSUPPORTED_DTYPE, "unsupported tensor dtype: " + std::to_string(info.dtype)};
            ok = false;
        }
        // ModelLoadError::TensorDataError(format!("{}: {e}", name)), src/lib.rs:133
        if (!ok) return fail(TIR_ERR_TENSOR_DATA, "Tensor Weight Data Load Error: " + info.name + ": " + te.msg);
        info.data = map + toff;
        info.data_bytes = bytes;
        g->index[info.name] = ti;
    }

    // Sizes the reference hard-codes, read from the tensors when present.
    t.kv_dim = t.k_v_heads * t.dim;
    if (const TensorInfo* ti = gguf_find(g, "blk.0.ffn_gate.weight"))
        if (ti->shape.size() >= 2) t.ffn_dim = ti->shape[1];
    if (const TensorInfo* ti = gguf_find(g, "output.weight"))
        if (ti->shape.size() >= 2) t.vocab = ti->shape[1];
    t.mode = 0;
    g->transformer = t;
    g->has_transformer = true;
    return TIR_OK;
}

}  // namespace tir
