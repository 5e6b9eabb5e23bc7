// tokenizer.cpp -- the reference's text layer on the host: BPE encode and
// decode (src/tokenizer.rs:37-150) over the GGUF's tokenizer.ggml.tokens and
// tokenizer.ggml.merges, and the text entry points of its drivers
// (generate / generate_capped, src/lib.rs:140-314) on the device decode loop.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "host.h"

struct tir_tokenizer {
    std::vector<std::string> vocab;  // id -> token ("" for a non-string item)
    std::vector<bool> is_str;        // the item at id is a string
    // Rust HashMap::insert overwrites: a repeated token maps to its last id,
    // a repeated merge to its last rank.
    std::unordered_map<std::string, int64_t> vocab_map;
    std::unordered_map<std::string, int64_t> merge_rank;
};

namespace tir {
namespace {

const char kLowerOneEighthBlock[] = "\xE2\x96\x81";  // U+2581, sentencepiece's space

// Length of the UTF-8 character starting at s[i] in a valid string.
size_t utf8_len(unsigned char b) {
    if (b < 0x80) return 1;
    if (b >= 0xF0) return 4;
    if (b >= 0xE0) return 3;
    return 2;
}

// The text is a Rust &str in the reference: valid UTF-8 is a precondition.
bool valid_utf8(const std::string& s) {
    size_t i = 0;
    while (i < s.size()) {
        const unsigned char b = static_cast<unsigned char>(s[i]);
        size_t n = 0;
        unsigned char lo = 0x80, hi = 0xBF;
        if (b < 0x80) {
            ++i;
            continue;
        } else if (b >= 0xC2 && b <= 0xDF) {
            n = 1;
        } else if (b == 0xE0) {
            n = 2;
            lo = 0xA0;
        } else if (b >= 0xE1 && b <= 0xEC) {
            n = 2;
        } else if (b == 0xED) {
            n = 2;
            hi = 0x9F;
        } else if (b >= 0xEE && b <= 0xEF) {
            n = 2;
        } else if (b == 0xF0) {
            n = 3;
            lo = 0x90;
        } else if (b >= 0xF1 && b <= 0xF3) {
            n = 3;
        } else if (b == 0xF4) {
            n = 3;
            hi = 0x8F;
        } else {
            return false;
        }
        for (size_t k = 1; k <= n; ++k) {
            if (i + k >= s.size()) return false;
            const unsigned char c = static_cast<unsigned char>(s[i + k]);
            const unsigned char l = k == 1 ? lo : 0x80, h = k == 1 ? hi : 0xBF;
            if (c < l || c > h) return false;
        }
        i += n + 1;
    }
    return true;
}

// String::from_utf8_lossy: valid sequences kept, each maximal ill-formed
// subpart replaced by one U+FFFD.
std::string from_utf8_lossy(const std::string& s) {
    static const char kRepl[] = "\xEF\xBF\xBD";
    std::string out;
    out.reserve(s.size());
    size_t i = 0;
    while (i < s.size()) {
        const unsigned char b = static_cast<unsigned char>(s[i]);
        if (b < 0x80) {
            out.push_back(static_cast<char>(b));
            ++i;
            continue;
        }
        size_t n = 0;
        unsigned char lo = 0x80, hi = 0xBF;
        if (b >= 0xC2 && b <= 0xDF) {
            n = 1;
        } else if (b == 0xE0) {
            n = 2;
            lo = 0xA0;
        } else if (b >= 0xE1 && b <= 0xEC) {
            n = 2;
        } else if (b == 0xED) {
            n = 2;
            hi = 0x9F;
        } else if (b >= 0xEE && b <= 0xEF) {
            n = 2;
        } else if (b == 0xF0) {
            n = 3;
            lo = 0x90;
        } else if (b >= 0xF1 && b <= 0xF3) {
            n = 3;
        } else if (b == 0xF4) {
            n = 3;
            hi = 0x8F;
        } else {
            out += kRepl;  // never a lead byte
            ++i;
            continue;
        }
        size_t k = 1;
        for (; k <= n && i + k < s.size(); ++k) {
            const unsigned char c = static_cast<unsigned char>(s[i + k]);
            const unsigned char l = k == 1 ? lo : 0x80, h = k == 1 ? hi : 0xBF;
            if (c < l || c > h) break;
        }
        if (k == n + 1) {
            out.append(s, i, n + 1);
            i += n + 1;
        } else {
            out += kRepl;  // the lead and the continuation bytes that fit it
            i += k;
        }
    }
    return out;
}

// parse_byte_token (src/tokenizer.rs:145-150): "<0x" hex ">" with the hex
// part parsed by u8::from_str_radix(_, 16) (an optional '+', then hex
// digits, value <= 255).
bool parse_byte_token(const std::string& t, unsigned char* out) {
    if (t.size() < 4 || t.compare(0, 3, "<0x") != 0 || t.back() != '>') return false;
    std::string h = t.substr(3, t.size() - 4);
    if (!h.empty() && h[0] == '+') h.erase(0, 1);
    if (h.empty()) return false;
    unsigned v = 0;
    for (char c : h) {
        unsigned d;
        if (c >= '0' && c <= '9')
            d = static_cast<unsigned>(c - '0');
        else if (c >= 'a' && c <= 'f')
            d = static_cast<unsigned>(c - 'a' + 10);
        else if (c >= 'A' && c <= 'F')
            d = static_cast<unsigned>(c - 'A' + 10);
        else
            return false;
        v = v * 16 + d;
        if (v > 255) return false;
    }
    *out = static_cast<unsigned char>(v);
    return true;
}

tir_status build(const std::vector<std::string>& tokens, const std::vector<bool>& is_str,
                 const std::vector<std::string>& merges, const std::vector<bool>& merge_is_str, tir_tokenizer** out) {
    tir_tokenizer* t = new tir_tokenizer;
    t->vocab = tokens;
    t->is_str = is_str;
    for (size_t id = 0; id < tokens.size(); ++id)
        if (is_str[id]) t->vocab_map[tokens[id]] = static_cast<int64_t>(id);
    for (size_t r = 0; r < merges.size(); ++r)
        if (merge_is_str[r]) t->merge_rank[merges[r]] = static_cast<int64_t>(r);
    *out = t;
    return TIR_OK;
}

// encode (src/tokenizer.rs:37-120).
std::vector<int32_t> encode(const tir_tokenizer* t, const std::string& text) {
    // 1. normalize: a leading space, every ' ' -> U+2581
    std::string norm;
    const std::string spaced = " " + text;
    for (char c : spaced) {
        if (c == ' ')
            norm += kLowerOneEighthBlock;
        else
            norm.push_back(c);
    }
    // 2. one symbol per character
    std::vector<std::string> sym;
    for (size_t i = 0; i < norm.size();) {
        const size_t n = utf8_len(static_cast<unsigned char>(norm[i]));
        sym.emplace_back(norm, i, n);
        i += n;
    }
    // 3. merge the best-ranked adjacent pair (the first of equal rank) until none
    std::string key;
    for (;;) {
        int64_t best_rank = -1;
        size_t best_i = 0;
        for (size_t i = 0; i + 1 < sym.size(); ++i) {
            key.assign(sym[i]);
            key.push_back(' ');
            key.append(sym[i + 1]);
            const auto it = t->merge_rank.find(key);
            if (it != t->merge_rank.end() && (best_rank < 0 || it->second < best_rank)) {
                best_rank = it->second;
                best_i = i;
            }
        }
        if (best_rank < 0) break;
        sym[best_i] += sym[best_i + 1];
        sym.erase(sym.begin() + static_cast<std::ptrdiff_t>(best_i) + 1);
    }
    // BOS (id 1, as the reference hard-codes), then each symbol's id, or its
    // bytes as <0xXX> tokens (unk 0 when even those are missing)
    std::vector<int32_t> ids{1};
    char bt[8];
    for (const std::string& s : sym) {
        const auto it = t->vocab_map.find(s);
        if (it != t->vocab_map.end()) {
            ids.push_back(static_cast<int32_t>(it->second));
            continue;
        }
        for (unsigned char b : s) {
            std::snprintf(bt, sizeof(bt), "<0x%02X>", b);
            const auto jt = t->vocab_map.find(bt);
            ids.push_back(jt != t->vocab_map.end() ? static_cast<int32_t>(jt->second) : 0);
        }
    }
    return ids;
}

// decode (src/tokenizer.rs:122-143); false with *bad = the id on UnknownId.
bool decode(const tir_tokenizer* t, const int32_t* ids, int64_t n, std::string* out, int64_t* bad) {
    std::string bytes;
    for (int64_t i = 0; i < n; ++i) {
        const int64_t id = ids[i];
        if (id < 0 || id >= static_cast<int64_t>(t->vocab.size()) || !t->is_str[static_cast<size_t>(id)]) {
            *bad = id;
            return false;
        }
        const std::string& tok = t->vocab[static_cast<size_t>(id)];
        unsigned char b;
        if (parse_byte_token(tok, &b)) {
            bytes.push_back(static_cast<char>(b));
        } else {
            for (size_t k = 0; k < tok.size();) {
                if (tok.compare(k, 3, kLowerOneEighthBlock) == 0) {
                    bytes.push_back(' ');
                    k += 3;
                } else {
                    bytes.push_back(tok[k++]);
                }
            }
        }
    }
    *out = from_utf8_lossy(bytes);
    return true;
}

tir_status copy_text(const std::string& s, char* out, int64_t cap, int64_t* len) {
    if (len) *len = static_cast<int64_t>(s.size());
    if (out && cap > 0) {
        const size_t n = std::min(static_cast<size_t>(cap - 1), s.size());
        std::memcpy(out, s.data(), n);
        out[n] = '\0';
    }
    return TIR_OK;
}

tir_status copy_ids(const std::vector<int32_t>& v, int32_t* out, int64_t cap, int64_t* n) {
    if (n) *n = static_cast<int64_t>(v.size());
    if (out && cap > 0) std::memcpy(out, v.data(), std::min(static_cast<size_t>(cap), v.size()) * sizeof(int32_t));
    return TIR_OK;
}

}  // namespace
}  // namespace tir

using namespace tir;

extern "C" {

tir_status tir_tokenizer_create(const tir_gguf* g, tir_tokenizer** out) {
    clear_error();
    if (!g || !out) return fail(TIR_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    // the last field of each name counts, as in the drivers' scan (src/lib.rs:149-157)
    const MetaField* tokens = nullptr;
    const MetaField* merges = nullptr;
    for (const MetaField& f : g->fields) {
        if (f.name == "tokenizer.ggml.tokens") tokens = &f;
        if (f.name == "tokenizer.ggml.merges") merges = &f;
    }
    if (!tokens) return fail(TIR_ERR_MISSING_FIELD, "missing required field: ggml.tokens");
    if (!merges) return fail(TIR_ERR_MISSING_FIELD, "missing required field: ggml.merges");
    if (tokens->value.vtype != TIR_GGUF_ARRAY)
        return fail(TIR_ERR_WRONG_TYPE, "tokenizer field has wrong type; expected array of tokens");
    if (merges->value.vtype != TIR_GGUF_ARRAY)
        return fail(TIR_ERR_WRONG_TYPE, "tokenizer field has wrong type; expected array of merges");
    std::vector<std::string> tv, mv;
    std::vector<bool> ts, ms;
    for (const MetaValue& v : tokens->value.items) {
        ts.push_back(v.vtype == TIR_GGUF_STRING);
        tv.push_back(v.vtype == TIR_GGUF_STRING ? v.str : std::string());
    }
    for (const MetaValue& v : merges->value.items) {
        ms.push_back(v.vtype == TIR_GGUF_STRING);
        mv.push_back(v.vtype == TIR_GGUF_STRING ? v.str : std::string());
    }
    return build(tv, ts, mv, ms, out);
}

tir_status tir_tokenizer_create_from(const char* const* tokens, const uint64_t* token_lens, int64_t n_tokens,
                                     const char* const* merges, const uint64_t* merge_lens, int64_t n_merges,
                                     tir_tokenizer** out) {
    clear_error();
    if (!out || n_tokens < 0 || n_merges < 0 || (n_tokens > 0 && (!tokens || !token_lens)) ||
        (n_merges > 0 && (!merges || !merge_lens)))
        return fail(TIR_ERR_INVALID_ARG, "null argument or negative count");
    *out = nullptr;
    std::vector<std::string> tv, mv;
    for (int64_t i = 0; i < n_tokens; ++i) tv.emplace_back(tokens[i], token_lens[i]);
    for (int64_t i = 0; i < n_merges; ++i) mv.emplace_back(merges[i], merge_lens[i]);
    return build(tv, std::vector<bool>(tv.size(), true), mv, std::vector<bool>(mv.size(), true), out);
}

void tir_tokenizer_destroy(tir_tokenizer* t) { delete t; }

int64_t tir_tokenizer_vocab_size(const tir_tokenizer* t) { return t ? static_cast<int64_t>(t->vocab.size()) : 0; }

tir_status tir_encode(const tir_tokenizer* t, const char* text, int64_t text_len, int32_t* ids, int64_t cap,
                      int64_t* n) {
    clear_error();
    if (!t || (!text && text_len > 0) || text_len < 0) return fail(TIR_ERR_INVALID_ARG, "null argument");
    const std::string s(text ? text : "", static_cast<size_t>(text_len));
    if (!valid_utf8(s)) return fail(TIR_ERR_INVALID_UTF8, "text is not valid UTF-8");
    return copy_ids(encode(t, s), ids, cap, n);
}

tir_status tir_decode(const tir_tokenizer* t, const int32_t* ids, int64_t n_ids, char* out, int64_t cap,
                      int64_t* len) {
    clear_error();
    if (!t || (!ids && n_ids > 0) || n_ids < 0) return fail(TIR_ERR_INVALID_ARG, "null argument");
    std::string s;
    int64_t bad = 0;
    if (!decode(t, ids, n_ids, &s, &bad))
        return fail(TIR_ERR_BAD_TOKEN, "token id " + std::to_string(bad) + " is not in the vocab");
    return copy_text(s, out, cap, len);
}

}  // extern "C"
