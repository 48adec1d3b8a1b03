// tl_tokenizer.cpp -- the Mistral BPE tokenizer of the model binary, on the
// host (tokenizer.cpp:1-209 of the reference): Metaspace pre-tokenisation,
// UTF-8 chunking with <0xXX> byte fallback, repeated merging of the
// lowest-ranked adjacent pair, BOS prepended; decoding maps the stored
// pieces back with "▁" -> " ".  The reference's undefined cases (a byte
// fallback piece or <s> missing from the vocabulary, an id outside it, a
// vocabulary id past its size) return errors here.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "tl_common.cuh"
#include "tl_json.h"

using namespace tl;

struct tl_tokenizer {
    std::vector<std::string> id_to_token;
    std::unordered_map<std::string, uint32_t> token_to_id;
    std::unordered_map<uint64_t, uint32_t> merge_rank;  // packed (left, right) -> merge index
    std::unordered_map<uint64_t, uint32_t> merge_id;    // packed (left, right) -> merged token id
};

namespace {

const char kMeta[] = "\xE2\x96\x81";  // U+2581 "▁", the Metaspace marker (3 bytes)

uint64_t pack(uint32_t left, uint32_t right) { return (static_cast<uint64_t>(left) << 32) | right; }

// token_to_id[s] as the reference's operator[]: a missing piece is inserted with id 0.
uint32_t lookup_or_zero(tl_tokenizer* t, const std::string& s) { return t->token_to_id[s]; }

// Tokenizer::load (tokenizer.cpp:37-68) from the tokenizer object {vocab, merges}.
tl_status load_model(tl_tokenizer* t, const JValue& tok) {
    const JValue* vocab = tok.get("vocab");
    if (!vocab || vocab->type != JValue::Obj) return set_error(TL_ERR_FORMAT, "tokenizer: no \"vocab\" object");
    t->id_to_token.assign(vocab->obj.size(), std::string());
    for (const auto& kv : vocab->obj) {
        if (kv.second.type != JValue::Int || kv.second.i < 0 ||
            static_cast<uint64_t>(kv.second.i) >= t->id_to_token.size())
            return set_error(TL_ERR_FORMAT, "tokenizer: id of piece \"%s\" outside the vocabulary", kv.first.c_str());
        const uint32_t id = static_cast<uint32_t>(kv.second.i);
        t->id_to_token[id] = kv.first;
        t->token_to_id[kv.first] = id;
    }
    const JValue* merges = tok.get("merges");
    if (!merges || merges->type == JValue::Null) return TL_OK;
    if (merges->type != JValue::Arr) return set_error(TL_ERR_FORMAT, "tokenizer: \"merges\" is not an array");
    uint32_t i = 0;
    for (const JValue& item : merges->arr) {
        if (item.type != JValue::Str) return set_error(TL_ERR_FORMAT, "tokenizer: merge %u is not a string", i);
        const std::string& m = item.s;
        const size_t sp = m.find(' ');
        // as substr(0, s) / substr(s + 1): no space splits into the whole string twice
        const std::string a = m.substr(0, sp), b = m.substr(sp == std::string::npos ? 0 : sp + 1);
        const uint64_t p = pack(lookup_or_zero(t, a), lookup_or_zero(t, b));
        t->merge_rank[p] = i;
        t->merge_id[p] = lookup_or_zero(t, a + b);
        i++;
    }
    return TL_OK;
}

// Tokenizer::get_id (tokenizer.cpp:16-35): the piece, or its bytes as <0xXX> pieces.
tl_status get_id(const tl_tokenizer* t, const std::string& s, std::vector<uint32_t>& out) {
    const auto it = t->token_to_id.find(s);
    if (it != t->token_to_id.end()) {
        out.push_back(it->second);
        return TL_OK;
    }
    for (unsigned char c : s) {
        char buf[8];
        std::snprintf(buf, sizeof(buf), "<0x%02X>", c);
        const auto bit = t->token_to_id.find(buf);
        if (bit == t->token_to_id.end())
            return set_error(TL_ERR_FORMAT, "tokenizer: byte fallback piece %s is not in the vocabulary", buf);
        out.push_back(bit->second);
    }
    return TL_OK;
}

// Tokenizer::encode (tokenizer.cpp:121-177).
tl_status encode(const tl_tokenizer* t, const std::string& text, std::vector<uint32_t>& tokens) {
    std::string s = kMeta;  // pre_tokenize_mistral (tokenizer.cpp:108-119)
    for (char c : text) {
        if (c == ' ') s += kMeta;
        else s += c;
    }
    tokens.clear();
    for (size_t i = 0; i < s.size();) {
        const unsigned char b0 = static_cast<unsigned char>(s[i]);
        size_t len = 1;  // UTF-8 sequence length from the lead byte; anything else is one byte
        if ((b0 & 0x80) == 0x00) len = 1;
        else if ((b0 & 0xE0) == 0xC0) len = 2;
        else if ((b0 & 0xF0) == 0xE0) len = 3;
        else if ((b0 & 0xF8) == 0xF0) len = 4;
        TL_TRY(get_id(t, s.substr(i, len), tokens));
        i += len;
    }
    // merge the lowest-ranked adjacent pair (first occurrence), all its occurrences left to right
    for (;;) {
        uint32_t best = UINT32_MAX;
        uint64_t bp = UINT64_MAX;
        for (size_t i = 0; i + 1 < tokens.size(); i++) {
            const uint64_t p = pack(tokens[i], tokens[i + 1]);
            const auto it = t->merge_rank.find(p);
            if (it != t->merge_rank.end() && it->second < best) {
                best = it->second;
                bp = p;
            }
        }
        if (bp == UINT64_MAX) break;
        const uint32_t left = static_cast<uint32_t>(bp >> 32), right = static_cast<uint32_t>(bp);
        const uint32_t merged = t->merge_id.at(bp);
        std::vector<uint32_t> next;
        next.reserve(tokens.size());
        for (size_t i = 0; i < tokens.size();) {
            if (tokens[i] == left && i + 1 < tokens.size() && tokens[i + 1] == right) {
                next.push_back(merged);
                i += 2;
            } else {
                next.push_back(tokens[i++]);
            }
        }
        tokens.swap(next);
    }
    const auto bos = t->token_to_id.find("<s>");  // BOS (tokenizer.cpp:174)
    if (bos == t->token_to_id.end()) return set_error(TL_ERR_FORMAT, "tokenizer: no <s> piece for BOS");
    tokens.insert(tokens.begin(), bos->second);
    return TL_OK;
}

// Tokenizer::decode_mistral (tokenizer.cpp:179-201): every "▁" becomes " ".
std::string decode_piece(const std::string& s) {
    const size_t n = sizeof(kMeta) - 1;
    if (s.size() < n) return s;
    std::string r;
    size_t i = 0;
    while (i <= s.size() - n) {
        if (s.compare(i, n, kMeta) == 0) {
            r += ' ';
            i += n;
        } else {
            r += s[i++];
        }
    }
    if (i < s.size()) r += s.substr(i);
    return r;
}

// The "tokenizer" member of a model binary's header (export_mistral.py:143-150).
tl_status load_from_header(const uint8_t* data, size_t size, tl_tokenizer** out) {
    if (size < 8) return set_error(TL_ERR_FORMAT, "model binary shorter than its header size field");
    uint64_t hlen = 0;
    std::memcpy(&hlen, data, 8);
    if (hlen > size - 8) return set_error(TL_ERR_FORMAT, "header of %llu bytes past the end", (unsigned long long)hlen);
    // the header may be padded after the JSON text
    size_t jlen = static_cast<size_t>(hlen);
    while (jlen > 0 && (data[8 + jlen - 1] == 0 || data[8 + jlen - 1] == ' ' || data[8 + jlen - 1] == '\n')) jlen--;
    JValue root;
    std::string err;
    JsonParser parser(reinterpret_cast<const char*>(data + 8), jlen);
    if (!parser.parse(root, err)) return set_error(TL_ERR_FORMAT, "model header: %s", err.c_str());
    const JValue* tok = root.get("tokenizer");
    if (!tok || tok->type != JValue::Obj) return set_error(TL_ERR_FORMAT, "model header has no tokenizer");
    std::unique_ptr<tl_tokenizer> t(new tl_tokenizer());
    TL_TRY(load_model(t.get(), *tok));
    *out = t.release();
    return TL_OK;
}

}  // namespace

extern "C" {

tl_status tl_tokenizer_load(const char* path, tl_tokenizer** out) {
    clear_error();
    TL_REQUIRE(path && out, "tl_tokenizer_load: null argument");
    *out = nullptr;
    FILE* f = std::fopen(path, "rb");
    if (!f) return set_error(TL_ERR_IO, "cannot open %s", path);
    uint8_t head[8];
    if (std::fread(head, 1, 8, f) != 8) {
        std::fclose(f);
        return set_error(TL_ERR_FORMAT, "%s: no header size field", path);
    }
    uint64_t hlen = 0;
    std::memcpy(&hlen, head, 8);
    if (hlen > (1ull << 32)) {
        std::fclose(f);
        return set_error(TL_ERR_FORMAT, "%s: header of %llu bytes", path, (unsigned long long)hlen);
    }
    std::vector<uint8_t> buf(8 + hlen);  // the header only, not the weights
    std::memcpy(buf.data(), head, 8);
    const size_t got = std::fread(buf.data() + 8, 1, hlen, f);
    std::fclose(f);
    if (got != hlen) return set_error(TL_ERR_FORMAT, "%s: truncated header", path);
    return load_from_header(buf.data(), buf.size(), out);
}

tl_status tl_tokenizer_load_buffer(const void* data, size_t size, tl_tokenizer** out) {
    clear_error();
    TL_REQUIRE(data && out, "tl_tokenizer_load_buffer: null argument");
    *out = nullptr;
    return load_from_header(static_cast<const uint8_t*>(data), size, out);
}

tl_status tl_tokenizer_load_json(const char* json, size_t len, tl_tokenizer** out) {
    clear_error();
    TL_REQUIRE(json && out, "tl_tokenizer_load_json: null argument");
    *out = nullptr;
    JValue root;
    std::string err;
    JsonParser parser(json, len);
    if (!parser.parse(root, err)) return set_error(TL_ERR_FORMAT, "tokenizer JSON: %s", err.c_str());
    std::unique_ptr<tl_tokenizer> t(new tl_tokenizer());
    TL_TRY(load_model(t.get(), root));
    *out = t.release();
    return TL_OK;
}

tl_status tl_tokenizer_destroy(tl_tokenizer* t) {
    clear_error();
    delete t;
    return TL_OK;
}

tl_status tl_tokenizer_vocab_size(const tl_tokenizer* t, size_t* n) {
    clear_error();
    TL_REQUIRE(t && n, "tl_tokenizer_vocab_size: null argument");
    *n = t->id_to_token.size();
    return TL_OK;
}

tl_status tl_tokenizer_encode(const tl_tokenizer* t, const char* text, size_t len, uint32_t* ids, size_t cap,
                              size_t* n_out) {
    clear_error();
    TL_REQUIRE(t && (text || len == 0) && n_out && (ids || cap == 0), "tl_tokenizer_encode: bad arguments");
    std::vector<uint32_t> tokens;
    TL_TRY(encode(t, std::string(text ? text : "", len), tokens));
    *n_out = tokens.size();
    if (tokens.size() > cap)
        return set_error(TL_ERR_CAPACITY, "tl_tokenizer_encode: %zu ids, room for %zu", tokens.size(), cap);
    if (!tokens.empty()) std::memcpy(ids, tokens.data(), tokens.size() * sizeof(uint32_t));
    return TL_OK;
}

tl_status tl_tokenizer_decode(const tl_tokenizer* t, const uint32_t* ids, size_t n, char* out, size_t cap,
                              size_t* len_out) {
    clear_error();
    TL_REQUIRE(t && (ids || n == 0) && len_out && (out || cap == 0), "tl_tokenizer_decode: bad arguments");
    std::string r;
    for (size_t i = 0; i < n; i++) {
        if (ids[i] >= t->id_to_token.size())
            return set_error(TL_ERR_INVALID_ARGUMENT, "tl_tokenizer_decode: id %u outside the vocabulary of %zu",
                             ids[i], t->id_to_token.size());
        r += decode_piece(t->id_to_token[ids[i]]);
    }
    *len_out = r.size();
    if (r.size() + 1 > cap)
        return set_error(TL_ERR_CAPACITY, "tl_tokenizer_decode: %zu bytes (+ NUL), room for %zu", r.size(), cap);
    std::memcpy(out, r.data(), r.size());
    out[r.size()] = '\0';
    return TL_OK;
}

}  // extern "C"
