// pack.cu -- the reference's weight file (a pack, src/pack.rs) read on the host, and the two
// models loaded from one onto the device.
//
// A pack is "TELMOPAK", a little-endian u32 format version (1) and 4 zero bytes; the entries' data,
// each at a multiple of 64 bytes; a JSON index naming the model, its metadata and every entry; and
// a trailer of the index's offset and length (u64s) and "TELMOIDX". The index is checked as the
// reference checks it (Pack::parse, src/pack.rs:98-259) before any entry is used: known kinds and
// precisions, sizes that match the shapes, 64-byte aligned ranges inside the data section, no
// overlaps, unique names. Loading a model reads its config.json entry (Config::from_json,
// src/granite.rs:60-146, src/parakeet.rs:70-141), creates the model and uploads every entry it
// knows (the 8-bit matrices as they are stored; others are refused by the upload).
#include "../../include/telmo_b200.h"
#include "api_internal.h"
#include "granite_internal.h"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <utility>
#include <vector>

namespace telmo {

namespace {

thread_local std::string pack_error;

int fail_pack(const std::string& why) {
    pack_error = why;
    return TELMO_ERR_MODEL;
}

// ---- a small JSON reader (RFC 8259: objects, arrays, strings, numbers, true/false/null) --------

struct Json {
    enum Type { kNull, kBool, kNumber, kString, kArray, kObject } type = kNull;
    bool b = false;
    std::string text;  // a number's text, or a string's value
    std::vector<Json> items;
    std::vector<std::pair<std::string, Json>> members;

    const Json* get(const char* key) const {
        if (type != kObject) return nullptr;
        for (const auto& m : members)
            if (m.first == key) return &m.second;
        return nullptr;
    }
    // An unsigned integer written without sign, fraction or exponent.
    bool as_u64(uint64_t& out) const {
        if (type != kNumber || text.empty() || text.size() > 19) return false;
        uint64_t v = 0;
        for (char ch : text) {
            if (ch < '0' || ch > '9') return false;
            v = v * 10 + static_cast<uint64_t>(ch - '0');
        }
        out = v;
        return true;
    }
};

struct JsonParser {
    const char* p;
    const char* end;
    int depth = 0;

    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool literal(const char* s) {
        const size_t n = strlen(s);
        if (static_cast<size_t>(end - p) < n || memcmp(p, s, n)) return false;
        p += n;
        return true;
    }
    static void put_utf8(std::string& out, uint32_t c) {
        if (c < 0x80) {
            out += static_cast<char>(c);
        } else if (c < 0x800) {
            out += static_cast<char>(0xC0 | (c >> 6));
            out += static_cast<char>(0x80 | (c & 0x3F));
        } else if (c < 0x10000) {
            out += static_cast<char>(0xE0 | (c >> 12));
            out += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (c & 0x3F));
        } else {
            out += static_cast<char>(0xF0 | (c >> 18));
            out += static_cast<char>(0x80 | ((c >> 12) & 0x3F));
            out += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (c & 0x3F));
        }
    }
    bool hex4(uint32_t& v) {
        if (end - p < 4) return false;
        v = 0;
        for (int i = 0; i < 4; ++i) {
            const char ch = *p++;
            v <<= 4;
            if (ch >= '0' && ch <= '9') v |= static_cast<uint32_t>(ch - '0');
            else if (ch >= 'a' && ch <= 'f') v |= static_cast<uint32_t>(ch - 'a' + 10);
            else if (ch >= 'A' && ch <= 'F') v |= static_cast<uint32_t>(ch - 'A' + 10);
            else return false;
        }
        return true;
    }
    bool string(std::string& out) {
        if (p >= end || *p != '"') return false;
        ++p;
        while (p < end && *p != '"') {
            const unsigned char ch = static_cast<unsigned char>(*p++);
            if (ch < 0x20) return false;
            if (ch != '\\') {
                out += static_cast<char>(ch);
                continue;
            }
            if (p >= end) return false;
            const char e = *p++;
            switch (e) {
            case '"': out += '"'; break;
            case '\\': out += '\\'; break;
            case '/': out += '/'; break;
            case 'b': out += '\b'; break;
            case 'f': out += '\f'; break;
            case 'n': out += '\n'; break;
            case 'r': out += '\r'; break;
            case 't': out += '\t'; break;
            case 'u': {
                uint32_t c;
                if (!hex4(c)) return false;
                if (c >= 0xD800 && c < 0xDC00) {  // a surrogate pair
                    uint32_t lo;
                    if (end - p < 2 || p[0] != '\\' || p[1] != 'u') return false;
                    p += 2;
                    if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                    c = 0x10000 + ((c - 0xD800) << 10) + (lo - 0xDC00);
                } else if (c >= 0xDC00 && c < 0xE000) {
                    return false;
                }
                put_utf8(out, c);
                break;
            }
            default: return false;
            }
        }
        if (p >= end) return false;
        ++p;
        return true;
    }
    bool number(std::string& out) {
        const char* s = p;
        if (p < end && *p == '-') ++p;
        if (p >= end) return false;
        if (*p == '0') {
            ++p;
        } else if (*p >= '1' && *p <= '9') {
            while (p < end && *p >= '0' && *p <= '9') ++p;
        } else {
            return false;
        }
        if (p < end && *p == '.') {
            ++p;
            if (p >= end || *p < '0' || *p > '9') return false;
            while (p < end && *p >= '0' && *p <= '9') ++p;
        }
        if (p < end && (*p == 'e' || *p == 'E')) {
            ++p;
            if (p < end && (*p == '+' || *p == '-')) ++p;
            if (p >= end || *p < '0' || *p > '9') return false;
            while (p < end && *p >= '0' && *p <= '9') ++p;
        }
        out.assign(s, p);
        return true;
    }
    bool value(Json& v) {
        if (++depth > 128) return false;
        ws();
        if (p >= end) return false;
        bool ok = true;
        if (*p == '{') {
            ++p;
            v.type = Json::kObject;
            ws();
            if (p < end && *p == '}') {
                ++p;
            } else {
                for (;;) {
                    ws();
                    std::string key;
                    if (!string(key)) { ok = false; break; }
                    ws();
                    if (p >= end || *p != ':') { ok = false; break; }
                    ++p;
                    Json item;
                    if (!value(item)) { ok = false; break; }
                    v.members.emplace_back(std::move(key), std::move(item));
                    ws();
                    if (p < end && *p == ',') { ++p; continue; }
                    if (p < end && *p == '}') { ++p; break; }
                    ok = false;
                    break;
                }
            }
        } else if (*p == '[') {
            ++p;
            v.type = Json::kArray;
            ws();
            if (p < end && *p == ']') {
                ++p;
            } else {
                for (;;) {
                    Json item;
                    if (!value(item)) { ok = false; break; }
                    v.items.push_back(std::move(item));
                    ws();
                    if (p < end && *p == ',') { ++p; continue; }
                    if (p < end && *p == ']') { ++p; break; }
                    ok = false;
                    break;
                }
            }
        } else if (*p == '"') {
            v.type = Json::kString;
            ok = string(v.text);
        } else if (literal("true")) {
            v.type = Json::kBool;
            v.b = true;
        } else if (literal("false")) {
            v.type = Json::kBool;
        } else if (literal("null")) {
            v.type = Json::kNull;
        } else {
            v.type = Json::kNumber;
            ok = number(v.text);
        }
        --depth;
        return ok;
    }
};

bool parse_json(const char* data, size_t len, Json& out) {
    JsonParser ps{data, data + len};
    if (!ps.value(out)) return false;
    ps.ws();
    return ps.p == ps.end;
}

// ---- the pack ------------------------------------------------------------------------------

constexpr size_t kPrefix = 16, kTrailer = 24, kAlign = 64;
constexpr uint64_t kMaxIndex = 64ull << 20;

size_t round_up_64(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

int precision_of(const std::string& name) {
    if (name == "f32") return TELMO_PRECISION_F32;
    if (name == "f16") return TELMO_PRECISION_F16;
    if (name == "bf16") return TELMO_PRECISION_BF16;
    if (name == "int8") return TELMO_PRECISION_INT8;
    if (name == "q8_0") return TELMO_PRECISION_Q8_0;
    return -1;
}

size_t value_bytes(int precision) {
    return precision == TELMO_PRECISION_F32 ? 4 : (precision == TELMO_PRECISION_F16 || precision == TELMO_PRECISION_BF16) ? 2 : 1;
}

size_t scale_count(int precision, size_t n, size_t k) {
    const size_t panels = (n + 15) / 16;
    if (precision == TELMO_PRECISION_INT8) return panels * 16;
    if (precision == TELMO_PRECISION_Q8_0) return panels * ((k + 31) / 32) * 16;
    return 0;
}

}  // namespace

struct PackEntry {
    std::string name;
    int kind = TELMO_PACK_BYTES;
    int precision = -1;
    size_t n = 0, k = 0;
    std::vector<size_t> shape;
    size_t offset = 0, bytes = 0, scales_offset = 0, scales_bytes = 0;
    size_t lo_offset = 0, lo_bytes = 0;  // a device entry's low level (Q8_0)
};

}  // namespace telmo

using namespace telmo;

struct telmo_pack {
    std::vector<uint8_t> data;
    std::string model;
    std::vector<std::pair<std::string, std::string>> metadata;
    std::vector<PackEntry> entries;
    std::map<std::string, size_t> by_name;

    const PackEntry* find(const std::string& name) const {
        auto it = by_name.find(name);
        return it == by_name.end() ? nullptr : &entries[it->second];
    }
};

namespace {

int parse_pack(telmo_pack& pk) {
    // Pack::parse (src/pack.rs:98-259).
    const std::vector<uint8_t>& d = pk.data;
    const size_t len = d.size();
    if (len < kPrefix + kTrailer || memcmp(d.data(), "TELMOPAK", 8)) return fail_pack("It isn't a pack.");
    uint32_t version;
    memcpy(&version, d.data() + 8, 4);
    if (version != 1) {
        char buf[160];
        snprintf(buf, sizeof buf, "The pack has format version %u, and this build reads 1. Convert the model again.", version);
        return fail_pack(buf);
    }
    const uint8_t* trailer = d.data() + len - kTrailer;
    if (memcmp(trailer + 16, "TELMOIDX", 8)) return fail_pack("Its index is missing, so the file may be cut short.");
    uint64_t index_at, index_len;
    memcpy(&index_at, trailer, 8);
    memcpy(&index_len, trailer + 8, 8);
    if (index_len > kMaxIndex || index_at < kPrefix || index_at + index_len != len - kTrailer)
        return fail_pack("Its index is out of place.");
    Json root;
    if (!parse_json(reinterpret_cast<const char*>(d.data()) + index_at, static_cast<size_t>(index_len), root) ||
        root.type != Json::kObject)
        return fail_pack("Its index isn't valid JSON.");
    const Json* model = root.get("model");
    if (!model || model->type != Json::kString) return fail_pack("The index names no model.");
    pk.model = model->text;
    if (const Json* meta = root.get("metadata")) {
        if (meta->type == Json::kObject)
            for (const auto& m : meta->members) {
                if (m.second.type != Json::kString) return fail_pack("A metadata value isn't a string.");
                pk.metadata.emplace_back(m.first, m.second.text);
            }
    }
    const Json* list = root.get("entries");
    if (!list || list->type != Json::kArray) return fail_pack("The index lists no entries.");
    std::vector<std::pair<size_t, size_t>> ranges;
    for (const Json& item : list->items) {
        PackEntry e;
        const Json* name = item.get("name");
        if (!name || name->type != Json::kString) return fail_pack("An entry has no name.");
        e.name = name->text;
        auto num = [&](const char* key, size_t& out) -> int {
            uint64_t v;
            const Json* x = item.get(key);
            if (!x || !x->as_u64(v) || v >= (1ull << 40)) return fail_pack("Entry " + e.name + " has no valid " + key + ".");
            out = static_cast<size_t>(v);
            return TELMO_OK;
        };
        const Json* type = item.get("type");
        const std::string t = type && type->type == Json::kString ? type->text : "";
        size_t expected = 0;
        if (t == "matrix") {
            e.kind = TELMO_PACK_MATRIX;
            const Json* pr = item.get("precision");
            e.precision = pr && pr->type == Json::kString ? precision_of(pr->text) : -1;
            if (e.precision < 0) return fail_pack("Entry " + e.name + " has an unknown precision.");
            if (int rc = num("n", e.n)) return rc;
            if (int rc = num("k", e.k)) return rc;
            if (e.n == 0 || e.k == 0 || e.n > (1u << 24) || e.k > (1u << 24) ||
                (e.precision == TELMO_PRECISION_Q8_0 && e.k % 32))
                return fail_pack("Entry " + e.name + " has an impossible shape.");
            expected = (e.n + 15) / 16 * e.k * 16 * value_bytes(e.precision);
        } else if (t == "f32") {
            e.kind = TELMO_PACK_F32;
            const Json* shape = item.get("shape");
            if (!shape || shape->type != Json::kArray || shape->items.size() > 8)
                return fail_pack("Entry " + e.name + " has no valid shape.");
            expected = 4;
            for (const Json& dim : shape->items) {
                uint64_t v;
                if (!dim.as_u64(v) || v >= (1ull << 40)) return fail_pack("Entry " + e.name + " has no valid shape.");
                e.shape.push_back(static_cast<size_t>(v));
                if (v && expected > SIZE_MAX / v) return fail_pack("Entry " + e.name + " has the wrong size.");
                expected *= static_cast<size_t>(v);
            }
        } else if (t == "device") {
            // This build's extension (the reference has no such kind): an 8-bit matrix already in
            // the device layout -- n rows of round_up(k, 16) values, n row scales, and for Q8_0 a
            // low level of rows -- so loading it copies instead of repacking panels.
            e.kind = TELMO_PACK_DEVICE;
            const Json* pr = item.get("precision");
            e.precision = pr && pr->type == Json::kString ? precision_of(pr->text) : -1;
            if (e.precision != TELMO_PRECISION_INT8 && e.precision != TELMO_PRECISION_Q8_0)
                return fail_pack("Entry " + e.name + " has a precision the device layout doesn't hold.");
            if (int rc = num("n", e.n)) return rc;
            if (int rc = num("k", e.k)) return rc;
            if (e.n == 0 || e.k == 0 || e.n > (1u << 24) || e.k > (1u << 24) ||
                (e.precision == TELMO_PRECISION_Q8_0 && e.k % 32))
                return fail_pack("Entry " + e.name + " has an impossible shape.");
            expected = e.n * ((e.k + 15) / 16 * 16);
        } else if (t == "bytes") {
            e.kind = TELMO_PACK_BYTES;
        } else {
            return fail_pack("Entry " + e.name + " has an unknown type.");
        }
        if (int rc = num("offset", e.offset)) return rc;
        if (int rc = num("bytes", e.bytes)) return rc;
        if (e.kind != TELMO_PACK_BYTES && expected != e.bytes) return fail_pack("Entry " + e.name + " has the wrong size.");
        auto check_range = [&](size_t off, size_t bytes) -> int {
            if (off < kPrefix || off % kAlign || off + bytes < off || off + bytes > index_at)
                return fail_pack("Entry " + e.name + " is out of place.");
            ranges.emplace_back(off, off + bytes);
            return TELMO_OK;
        };
        if (int rc = check_range(e.offset, e.bytes)) return rc;
        if (e.kind == TELMO_PACK_MATRIX && scale_count(e.precision, e.n, e.k) > 0) {
            if (int rc = num("scales_bytes", e.scales_bytes)) return rc;
            if (e.scales_bytes != scale_count(e.precision, e.n, e.k) * 4)
                return fail_pack("Entry " + e.name + " has the wrong number of scales.");
            if (int rc = num("scales_offset", e.scales_offset)) return rc;
            if (int rc = check_range(e.scales_offset, e.scales_bytes)) return rc;
        }
        if (e.kind == TELMO_PACK_DEVICE) {
            if (int rc = num("scales_bytes", e.scales_bytes)) return rc;
            if (e.scales_bytes != e.n * 4) return fail_pack("Entry " + e.name + " has the wrong number of scales.");
            if (int rc = num("scales_offset", e.scales_offset)) return rc;
            if (int rc = check_range(e.scales_offset, e.scales_bytes)) return rc;
            if (e.precision == TELMO_PRECISION_Q8_0) {
                if (int rc = num("lo_bytes", e.lo_bytes)) return rc;
                if (e.lo_bytes != e.bytes) return fail_pack("Entry " + e.name + " has the wrong size.");
                if (int rc = num("lo_offset", e.lo_offset)) return rc;
                if (int rc = check_range(e.lo_offset, e.lo_bytes)) return rc;
            }
        }
        if (pk.by_name.count(e.name)) return fail_pack("Two entries are named " + e.name + ".");
        pk.by_name[e.name] = pk.entries.size();
        pk.entries.push_back(std::move(e));
    }
    std::sort(ranges.begin(), ranges.end());
    for (size_t i = 1; i < ranges.size(); ++i)
        if (ranges[i].first < ranges[i - 1].second) return fail_pack("Two entries overlap.");
    return TELMO_OK;
}

int make_pack(std::vector<uint8_t>&& data, telmo_pack** out) {
    auto* pk = new telmo_pack();
    pk->data = std::move(data);
    if (int rc = parse_pack(*pk)) {
        delete pk;
        return rc;
    }
    *out = pk;
    return TELMO_OK;
}

// ---- config.json ------------------------------------------------------------------------------

struct ConfigReader {
    const Json& root;
    const Json* enc = nullptr;
    std::string why;
    bool num(const Json* v, const char* key, int& out) {
        uint64_t x;
        const Json* j = v ? v->get(key) : nullptr;
        if (!j || !j->as_u64(x) || x > (1u << 30)) {
            why = std::string(key) + " is missing.";
            return false;
        }
        out = static_cast<int>(x);
        return true;
    }
    // The value as the reference compares it: a string, true/false, or a number's text; a
    // missing key takes the default (or fails without one).
    bool expect(const Json* v, const char* key, const char* want, const char* fallback = nullptr) {
        const Json* j = v ? v->get(key) : nullptr;
        std::string got;
        bool have = true;
        if (!j) {
            if (fallback) got = fallback;
            else have = false;
        } else if (j->type == Json::kString || j->type == Json::kNumber) {
            got = j->text;
        } else if (j->type == Json::kBool) {
            got = j->b ? "true" : "false";
        } else {
            have = false;
        }
        if (!have || got != want) {
            why = std::string(key) + " isn't " + want + ".";
            return false;
        }
        return true;
    }
};

int granite_config_from_json(const char* text, size_t len, telmo_granite_config* cfg) {
    // Config::from_json (src/granite.rs:60-146).
    Json root;
    const std::string pre = "config.json doesn't describe a supported Granite Speech CTC model. ";
    if (!parse_json(text, len, root)) return fail_pack(pre + "It isn't valid JSON.");
    ConfigReader r{root};
    r.enc = root.get("encoder_config");
    if (!r.enc) return fail_pack(pre + "It has no encoder_config.");
    const Json* enc = r.enc;
    if (!r.expect(&root, "model_type", "granite_speech5_ctc") || !r.expect(enc, "model_type", "granite_speech5_encoder") ||
        !r.expect(enc, "hidden_act", "silu", "silu") || !r.expect(enc, "attention_bias", "true", "true") ||
        !r.expect(&root, "tie_word_embeddings", "true", "true"))
        return fail_pack(pre + r.why);
    telmo_granite_config c{};
    int heads = 0, expansion = 0, enc_vocab = 0, kv = 0;
    if (!r.num(enc, "hidden_size", c.d_model) || !r.num(enc, "num_attention_heads", heads)) return fail_pack(pre + r.why);
    c.heads = heads;
    const Json* hd = enc->get("head_dim");
    if (!hd || hd->type == Json::kNull) c.head_dim = heads ? c.d_model / heads : 0;
    else if (!r.num(enc, "head_dim", c.head_dim)) return fail_pack(pre + r.why);
    const Json* kvj = enc->get("num_key_value_heads");
    if (!kvj || kvj->type == Json::kNull) kv = heads;
    else if (!r.num(enc, "num_key_value_heads", kv)) return fail_pack(pre + r.why);
    const Json* sub = enc->get("subsample_layers");
    if (!sub || sub->type == Json::kNull) {
        c.n_subsample = 2;
        c.subsample_layers[0] = 0;
        c.subsample_layers[1] = 1;
    } else {
        if (sub->type != Json::kArray || sub->items.size() > 8)
            return fail_pack(pre + "subsample_layers isn't a list of indices.");
        c.n_subsample = static_cast<int>(sub->items.size());
        for (size_t i = 0; i < sub->items.size(); ++i) {
            uint64_t v;
            if (!sub->items[i].as_u64(v) || v > 1024) return fail_pack(pre + "subsample_layers isn't a list of indices.");
            c.subsample_layers[i] = static_cast<int>(v);
        }
    }
    if (!r.num(enc, "num_hidden_layers", c.layers) || !r.num(enc, "intermediate_size", c.ff) ||
        !r.num(enc, "conv_kernel_size", c.conv_kernel) || !r.num(enc, "conv_expansion_factor", expansion) ||
        !r.num(enc, "num_mel_bins", c.n_mels) || !r.num(enc, "context_size", c.context) ||
        !r.num(enc, "max_position_embeddings", c.max_relative) || !r.num(&root, "vocab_size", c.vocab) ||
        !r.num(&root, "pad_token_id", c.blank) || !r.num(enc, "vocab_size", enc_vocab))
        return fail_pack(pre + r.why);
    c.conv_channels = c.d_model * expansion;
    bool bad = heads == 0 || kv != heads || heads * c.head_dim != c.d_model || c.head_dim % 16 || c.conv_kernel % 2 == 0 ||
               c.context == 0 || c.context > c.max_relative || c.layers < 2 || enc_vocab != c.vocab || c.blank >= c.vocab;
    for (int i = 0; i < c.n_subsample; ++i) {
        if (c.subsample_layers[i] >= c.layers) bad = true;
        if (i && c.subsample_layers[i] <= c.subsample_layers[i - 1]) bad = true;
    }
    if (bad) return fail_pack(pre + "Its sizes don't fit together.");
    *cfg = c;
    return TELMO_OK;
}

int parakeet_config_from_json(const char* text, size_t len, telmo_parakeet_config* cfg) {
    // Config::from_json (src/parakeet.rs:70-141).
    Json root;
    const std::string pre = "config.json doesn't describe a supported Parakeet TDT model. ";
    if (!parse_json(text, len, root)) return fail_pack(pre + "It isn't valid JSON.");
    ConfigReader r{root};
    r.enc = root.get("encoder_config");
    if (!r.enc) return fail_pack(pre + "It has no encoder_config.");
    const Json* enc = r.enc;
    if (!r.expect(&root, "model_type", "parakeet_tdt") || !r.expect(&root, "hidden_act", "relu") ||
        !r.expect(enc, "hidden_act", "silu") || !r.expect(enc, "attention_bias", "false") ||
        !r.expect(enc, "convolution_bias", "false") || !r.expect(enc, "scale_input", "false") ||
        !r.expect(enc, "subsampling_factor", "8") || !r.expect(enc, "subsampling_conv_kernel_size", "3") ||
        !r.expect(enc, "subsampling_conv_stride", "2"))
        return fail_pack(pre + r.why);
    const Json* durs = root.get("durations");
    if (!durs || durs->type != Json::kArray) return fail_pack(pre + "durations is missing.");
    telmo_parakeet_config c{};
    if (durs->items.size() > 8) return fail_pack(pre + "more than 8 durations.");
    c.n_durations = static_cast<int>(durs->items.size());
    for (size_t i = 0; i < durs->items.size(); ++i) {
        uint64_t v;
        if (!durs->items[i].as_u64(v) || v > 1024) return fail_pack(pre + "durations is missing.");
        c.durations[i] = static_cast<int>(v);
    }
    if (!r.num(enc, "hidden_size", c.d_model) || !r.num(enc, "num_attention_heads", c.heads) ||
        !r.num(enc, "num_hidden_layers", c.layers) || !r.num(enc, "intermediate_size", c.ff) ||
        !r.num(enc, "conv_kernel_size", c.conv_kernel) || !r.num(enc, "subsampling_conv_channels", c.sub_channels) ||
        !r.num(enc, "num_mel_bins", c.n_mels) || !r.num(&root, "decoder_hidden_size", c.pred_hidden) ||
        !r.num(&root, "num_decoder_layers", c.pred_layers) || !r.num(&root, "vocab_size", c.vocab) ||
        !r.num(&root, "blank_token_id", c.blank) || !r.num(&root, "max_symbols_per_step", c.max_symbols))
        return fail_pack(pre + r.why);
    if (c.blank + 1 != c.vocab || c.heads == 0 || c.d_model % c.heads || c.n_mels % 8 || c.conv_kernel % 2 == 0 ||
        c.n_durations == 0)
        return fail_pack(pre + "Its sizes don't fit together.");
    *cfg = c;
    return TELMO_OK;
}

const uint8_t* entry_data(const telmo_pack* pk, size_t off) { return pk->data.data() + off; }

// ---- writing packs ------------------------------------------------------------------------------

const char* precision_name(int precision) {
    switch (precision) {
        case TELMO_PRECISION_F32: return "f32";
        case TELMO_PRECISION_F16: return "f16";
        case TELMO_PRECISION_BF16: return "bf16";
        case TELMO_PRECISION_INT8: return "int8";
        default: return "q8_0";
    }
}

// A JSON string (RFC 8259 section 7): quotes, backslashes and control characters escaped; other
// bytes (UTF-8) as they are.
std::string json_string(const std::string& v) {
    std::string out = "\"";
    for (unsigned char ch : v) {
        if (ch == '"' || ch == '\\') {
            out += '\\';
            out += static_cast<char>(ch);
        } else if (ch < 0x20) {
            char buf[8];
            snprintf(buf, sizeof buf, "\\u%04x", ch);
            out += buf;
        } else {
            out += static_cast<char>(ch);
        }
    }
    return out + "\"";
}

}  // namespace

extern "C" int telmo_pack_from_bytes(const void* data, size_t len, telmo_pack** out) {
    if (!out || (!data && len)) return TELMO_ERR_ARGUMENT;
    *out = nullptr;
    const uint8_t* b = static_cast<const uint8_t*>(data);
    return make_pack(std::vector<uint8_t>(b, b + len), out);
}

extern "C" int telmo_pack_open(const char* path, telmo_pack** out) {
    if (!path || !out) return TELMO_ERR_ARGUMENT;
    *out = nullptr;
    FILE* f = fopen(path, "rb");
    if (!f) return fail_pack(std::string("Cannot open ") + path + ".");
    std::vector<uint8_t> data;
    if (fseek(f, 0, SEEK_END) == 0) {
        const long n = ftell(f);
        if (n > 0) {
            data.resize(static_cast<size_t>(n));
            fseek(f, 0, SEEK_SET);
            if (fread(data.data(), 1, data.size(), f) != data.size()) data.clear();
        }
    }
    fclose(f);
    return make_pack(std::move(data), out);
}

extern "C" void telmo_pack_free(telmo_pack* pk) { delete pk; }

extern "C" const char* telmo_pack_last_error(void) { return pack_error.c_str(); }

extern "C" const char* telmo_pack_model(const telmo_pack* pk) { return pk ? pk->model.c_str() : nullptr; }

extern "C" const char* telmo_pack_meta(const telmo_pack* pk, const char* key) {
    if (!pk || !key) return nullptr;
    for (const auto& m : pk->metadata)
        if (m.first == key) return m.second.c_str();
    return nullptr;
}

extern "C" size_t telmo_pack_entry_count(const telmo_pack* pk) { return pk ? pk->entries.size() : 0; }

extern "C" int telmo_pack_entry_info(const telmo_pack* pk, size_t i, const char** name, int* kind, int* precision,
                                     size_t* n, size_t* k, size_t* bytes) {
    if (!pk || i >= pk->entries.size()) return TELMO_ERR_ARGUMENT;
    const PackEntry& e = pk->entries[i];
    if (name) *name = e.name.c_str();
    if (kind) *kind = e.kind;
    if (precision) *precision = e.precision;
    if (n) *n = e.kind == TELMO_PACK_F32 ? (e.shape.empty() ? 1 : e.shape[0]) : e.n;
    if (k) *k = e.kind == TELMO_PACK_F32 ? (e.shape.size() > 1 ? e.bytes / 4 / std::max<size_t>(e.shape[0], 1) : 1) : e.k;
    if (bytes) *bytes = e.bytes;
    return TELMO_OK;
}

extern "C" int telmo_pack_bytes(const telmo_pack* pk, const char* name, const void** data, size_t* len) {
    if (!pk || !name || !data || !len) return TELMO_ERR_ARGUMENT;
    const PackEntry* e = pk->find(name);
    if (!e) return fail_pack(std::string("Entry ") + name + " is missing.");
    *data = entry_data(pk, e->offset);
    *len = e->bytes;
    return TELMO_OK;
}

extern "C" int telmo_pack_to_device(const telmo_pack* src, telmo_pack** out) {
    // Every Int8 and Q8_0 matrix re-encoded by the upload's own host routine (encode_device_rows),
    // so a model loaded from the result holds the same device bytes as one loaded from src. The
    // file is laid out first and written in place, in one allocation.
    if (!src || !out) return TELMO_ERR_ARGUMENT;
    *out = nullptr;
    std::vector<int> linear_perm;
    if (src->model == "parakeet-tdt") {
        const PackEntry* cj = src->find("config.json");
        if (!cj) return fail_pack("Entry config.json is missing.");
        telmo_parakeet_config cfg;
        if (int rc = parakeet_config_from_json(reinterpret_cast<const char*>(entry_data(src, cj->offset)), cj->bytes, &cfg))
            return rc;
        linear_perm = parakeet_linear_perm(cfg.sub_channels, cfg.n_mels);
    }
    // Layout: each entry's blobs (values; then scales; then a device entry's low level) at the
    // next 64-byte boundaries, and the index text that names them.
    struct Placed {
        int kind = TELMO_PACK_BYTES;
        size_t at = 0, bytes = 0, s_at = 0, s_bytes = 0, l_at = 0, l_bytes = 0;
    };
    std::vector<Placed> placed(src->entries.size());
    size_t end = kPrefix;
    auto place = [&](size_t bytes) {
        const size_t at = round_up_64(end);
        end = at + bytes;
        return at;
    };
    std::string index = "{\"model\":" + json_string(src->model) + ",\"metadata\":{";
    for (size_t i = 0; i < src->metadata.size(); ++i)
        index += (i ? "," : "") + json_string(src->metadata[i].first) + ":" + json_string(src->metadata[i].second);
    index += "},\"entries\":[";
    char buf[320];
    for (size_t i = 0; i < src->entries.size(); ++i) {
        const PackEntry& e = src->entries[i];
        Placed& pl = placed[i];
        index += (i ? ",{" : "{") + std::string("\"name\":") + json_string(e.name);
        const bool device = e.kind == TELMO_PACK_DEVICE ||
                            (e.kind == TELMO_PACK_MATRIX &&
                             (e.precision == TELMO_PRECISION_INT8 || e.precision == TELMO_PRECISION_Q8_0));
        if (device) {
            if (e.kind == TELMO_PACK_MATRIX && !linear_perm.empty() && e.name == "sub.linear" && linear_perm.size() != e.k)
                return fail_pack("Entry sub.linear doesn't fit config.json.");
            const size_t plane = e.n * ((e.k + 15) / 16 * 16);
            pl.kind = TELMO_PACK_DEVICE;
            pl.bytes = plane;
            pl.at = place(plane);
            pl.s_bytes = e.n * 4;
            pl.s_at = place(pl.s_bytes);
            snprintf(buf, sizeof buf,
                     ",\"type\":\"device\",\"precision\":\"%s\",\"n\":%zu,\"k\":%zu,\"offset\":%zu,\"bytes\":%zu,"
                     "\"scales_offset\":%zu,\"scales_bytes\":%zu",
                     precision_name(e.precision), e.n, e.k, pl.at, pl.bytes, pl.s_at, pl.s_bytes);
            index += buf;
            if (e.precision == TELMO_PRECISION_Q8_0) {
                pl.l_bytes = plane;
                pl.l_at = place(plane);
                snprintf(buf, sizeof buf, ",\"lo_offset\":%zu,\"lo_bytes\":%zu", pl.l_at, pl.l_bytes);
                index += buf;
            }
        } else if (e.kind == TELMO_PACK_MATRIX) {
            pl.kind = TELMO_PACK_MATRIX;
            pl.bytes = e.bytes;
            pl.at = place(e.bytes);
            snprintf(buf, sizeof buf, ",\"type\":\"matrix\",\"precision\":\"%s\",\"n\":%zu,\"k\":%zu,\"offset\":%zu,\"bytes\":%zu",
                     precision_name(e.precision), e.n, e.k, pl.at, pl.bytes);
            index += buf;
            if (e.scales_bytes) {
                pl.s_bytes = e.scales_bytes;
                pl.s_at = place(pl.s_bytes);
                snprintf(buf, sizeof buf, ",\"scales_offset\":%zu,\"scales_bytes\":%zu", pl.s_at, pl.s_bytes);
                index += buf;
            }
        } else if (e.kind == TELMO_PACK_F32) {
            pl.kind = TELMO_PACK_F32;
            pl.bytes = e.bytes;
            pl.at = place(e.bytes);
            index += ",\"type\":\"f32\",\"shape\":[";
            for (size_t d = 0; d < e.shape.size(); ++d) index += (d ? "," : "") + std::to_string(e.shape[d]);
            snprintf(buf, sizeof buf, "],\"offset\":%zu,\"bytes\":%zu", pl.at, pl.bytes);
            index += buf;
        } else {
            pl.bytes = e.bytes;
            pl.at = place(e.bytes);
            snprintf(buf, sizeof buf, ",\"type\":\"bytes\",\"offset\":%zu,\"bytes\":%zu", pl.at, pl.bytes);
            index += buf;
        }
        index += "}";
    }
    index += "]}";
    const uint64_t index_at = end, index_len = index.size();
    std::vector<uint8_t> data(end + index.size() + kTrailer, 0);
    memcpy(data.data(), "TELMOPAK", 8);
    const uint32_t version = 1;
    memcpy(data.data() + 8, &version, 4);
    uint8_t* d = data.data();
    for (size_t i = 0; i < src->entries.size(); ++i) {
        const PackEntry& e = src->entries[i];
        const Placed& pl = placed[i];
        if (pl.kind == TELMO_PACK_DEVICE && e.kind == TELMO_PACK_MATRIX) {
            const int* perm = !linear_perm.empty() && e.name == "sub.linear" ? linear_perm.data() : nullptr;
            encode_device_rows(e.precision, e.n, e.k, entry_data(src, e.offset),
                               reinterpret_cast<const float*>(entry_data(src, e.scales_offset)), perm,
                               reinterpret_cast<int8_t*>(d + pl.at), reinterpret_cast<int8_t*>(d + pl.l_at),
                               reinterpret_cast<float*>(d + pl.s_at));
            continue;
        }
        memcpy(d + pl.at, entry_data(src, e.offset), pl.bytes);
        if (pl.s_bytes) memcpy(d + pl.s_at, entry_data(src, e.scales_offset), pl.s_bytes);
        if (pl.l_bytes) memcpy(d + pl.l_at, entry_data(src, e.lo_offset), pl.l_bytes);
    }
    memcpy(d + index_at, index.data(), index.size());
    uint8_t* trailer = d + index_at + index_len;
    memcpy(trailer, &index_at, 8);
    memcpy(trailer + 8, &index_len, 8);
    memcpy(trailer + 16, "TELMOIDX", 8);
    return make_pack(std::move(data), out);
}

extern "C" int telmo_pack_save(const telmo_pack* pk, const char* path) {
    if (!pk || !path) return TELMO_ERR_ARGUMENT;
    FILE* f = fopen(path, "wb");
    if (!f) return fail_pack(std::string("Cannot create ") + path + ".");
    const bool ok = fwrite(pk->data.data(), 1, pk->data.size(), f) == pk->data.size();
    if (fclose(f) != 0 || !ok) return fail_pack(std::string("Cannot write ") + path + ".");
    return TELMO_OK;
}

extern "C" int telmo_granite_config_from_json(const char* json, size_t len, telmo_granite_config* out) {
    if (!json || !out) return TELMO_ERR_ARGUMENT;
    return granite_config_from_json(json, len, out);
}

extern "C" int telmo_parakeet_config_from_json(const char* json, size_t len, telmo_parakeet_config* out) {
    if (!json || !out) return TELMO_ERR_ARGUMENT;
    return parakeet_config_from_json(json, len, out);
}

namespace telmo {

int pack_load_entries(const telmo_pack* pk, const PackMatrixFn& set_matrix, const PackDeviceFn& set_device,
                      const PackVectorFn& set_vector, const PackKnowsFn& knows) {
    for (const PackEntry& e : pk->entries) {
        if (e.kind == TELMO_PACK_BYTES || !knows(e.name)) continue;
        if (e.kind == TELMO_PACK_MATRIX) {
            const float* scales = e.scales_bytes ? reinterpret_cast<const float*>(entry_data(pk, e.scales_offset)) : nullptr;
            if (int rc = set_matrix(e.name.c_str(), e.precision, e.n, e.k, entry_data(pk, e.offset), scales)) return rc;
        } else if (e.kind == TELMO_PACK_DEVICE) {
            const int8_t* lo = e.lo_bytes ? reinterpret_cast<const int8_t*>(entry_data(pk, e.lo_offset)) : nullptr;
            if (int rc = set_device(e.name.c_str(), e.precision, e.n, e.k,
                                    reinterpret_cast<const int8_t*>(entry_data(pk, e.offset)), lo,
                                    reinterpret_cast<const float*>(entry_data(pk, e.scales_offset))))
                return rc;
        } else {
            if (int rc = set_vector(e.name.c_str(), e.bytes / 4, reinterpret_cast<const float*>(entry_data(pk, e.offset))))
                return rc;
        }
    }
    return TELMO_OK;
}

}  // namespace telmo

extern "C" int telmo_granite_load_pack(telmo_ctx* ctx, const telmo_pack* pk, telmo_granite** out) {
    // Granite::from_pack (src/granite.rs:225-231, :424-500) onto the device.
    if (!ctx || !pk || !out) return TELMO_ERR_ARGUMENT;
    *out = nullptr;
    Ctx* c = as_ctx(ctx);
    if (pk->model != "granite-speech-ctc")
        return c->fail(TELMO_ERR_MODEL, "The pack holds %s, not Granite Speech.", pk->model.c_str());
    const PackEntry* cj = pk->find("config.json");
    if (!cj) return c->fail(TELMO_ERR_MODEL, "Entry config.json is missing.");
    telmo_granite_config cfg;
    if (granite_config_from_json(reinterpret_cast<const char*>(entry_data(pk, cj->offset)), cj->bytes, &cfg))
        return c->fail(TELMO_ERR_MODEL, "%s", pack_error.c_str());
    telmo_granite* g = nullptr;
    if (int rc = telmo_granite_create(ctx, &cfg, &g)) return rc;
    Granite* gm = reinterpret_cast<Granite*>(g);
    int rc = pack_load_entries(
        pk,
        [&](const char* name, int precision, size_t n, size_t k, const void* v, const float* s) {
            return telmo_granite_set_matrix(g, name, precision, n, k, v, s);
        },
        [&](const char* name, int precision, size_t n, size_t k, const int8_t* v, const int8_t* lo, const float* s) {
            return granite_set_device_matrix(g, name, precision, n, k, v, lo, s);
        },
        [&](const char* name, size_t len, const float* data) { return telmo_granite_set_vector(g, name, len, data); },
        [&](const std::string& name) {
            Granite::Entry e = gm->find(name);
            return e.mat != nullptr || e.vec != nullptr;
        });
    if (!rc) rc = telmo_granite_finalize(g);
    if (rc) {
        telmo_granite_free(g);
        return rc;
    }
    *out = g;
    return TELMO_OK;
}
