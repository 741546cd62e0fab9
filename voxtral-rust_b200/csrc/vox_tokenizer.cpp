// vox_tokenizer.cpp -- Tekken tokenizer decode (crates/voxtral/src/tokenizer.rs):
// the step after the token loop's argmax, turning ids into text.
//
// from_json_str (tokenizer.rs:72-130) reads tekken.json: config
// {default_vocab_size, default_num_special_tokens}, special_tokens [{rank,
// token_str, is_control}] (rank = id; ranks beyond the special count are
// skipped; missing ranks become "<missing-special-N>" control tokens), vocab
// [{rank, token_bytes (standard base64)}] (id = special count + rank; ids
// beyond default_vocab_size are skipped) and an optional audio block.  Field
// rules follow serde: required fields must be present with the right JSON
// type, unknown fields are ignored, usize fields take non-negative integers.
// The base64 alphabet is the standard one with canonical padding and no
// trailing bits, as base64 0.22's STANDARD engine decodes (Cargo.lock:99-100).
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/vox_decoder.h"
#include "vox_host.h"
#include "vox_json.h"

using namespace vox;

struct vox_tekken {
    size_t default_vocab_size = 0;
    size_t special_token_count = 0;
    std::vector<std::vector<uint8_t>> token_bytes;  // [default_vocab_size]
    std::vector<uint8_t> has_bytes;                 // Option<> flags of token_bytes
    struct Special {
        uint32_t id;
        std::string text;
        bool is_control;
    };
    std::vector<Special> specials;                  // [special_token_count]
    std::unordered_map<std::string, uint32_t> lookup;
    bool has_audio = false;
    vox_tekken_audio_config audio{};
};

namespace {

int b64_value(unsigned char c) {
    if (c >= 'A' && c <= 'Z') return c - 'A';
    if (c >= 'a' && c <= 'z') return c - 'a' + 26;
    if (c >= '0' && c <= '9') return c - '0' + 52;
    if (c == '+') return 62;
    if (c == '/') return 63;
    return -1;
}

// RFC 4648 section 4 decoding with canonical padding required and the unused
// low bits of the last symbol required to be zero.
bool b64_decode(const std::string& s, std::vector<uint8_t>* out) {
    out->clear();
    if (s.size() % 4) return false;
    for (size_t i = 0; i < s.size(); i += 4) {
        const bool last = i + 4 == s.size();
        int v[4];
        int pad = 0;
        for (int j = 0; j < 4; ++j) {
            const unsigned char c = (unsigned char)s[i + j];
            if (c == '=') {
                if (!last || j < 2) return false;
                v[j] = 0;
                ++pad;
            } else {
                if (pad) return false;  // data after padding
                v[j] = b64_value(c);
                if (v[j] < 0) return false;
            }
        }
        const uint32_t w = ((uint32_t)v[0] << 18) | ((uint32_t)v[1] << 12) | ((uint32_t)v[2] << 6) | (uint32_t)v[3];
        out->push_back((uint8_t)(w >> 16));
        if (pad == 2) {
            if (v[1] & 0x0F) return false;  // trailing bits
            continue;
        }
        out->push_back((uint8_t)(w >> 8));
        if (pad == 1) {
            if (v[2] & 0x03) return false;
            continue;
        }
        out->push_back((uint8_t)w);
    }
    return true;
}

bool get_usize(const Json& o, const char* key, size_t* out, std::string* err) {
    const Json* v = o.get(key);
    if (!v) {
        *err = std::string("missing field `") + key + "`";
        return false;
    }
    if (v->kind != Json::Number || !v->is_int || v->i64 < 0) {
        *err = std::string("invalid type for `") + key + "`, expected usize";
        return false;
    }
    *out = (size_t)v->i64;
    return true;
}

int parse(const char* json, size_t len, vox_tekken** out) {
    Json root;
    std::string err;
    JsonParser jp(json, len);
    if (!jp.parse(&root, &err)) return report_errorf(VOX_ERR_FORMAT, "parse tekken.json: %s", err.c_str());
    auto bad = [&](const std::string& m) { return report_errorf(VOX_ERR_FORMAT, "parse tekken.json: %s", m.c_str()); };
    if (root.kind != Json::Object) return bad("expected an object");
    const Json* cfg = root.get("config");
    const Json* vocab = root.get("vocab");
    const Json* specials = root.get("special_tokens");
    if (!cfg || cfg->kind != Json::Object) return bad("missing field `config`");
    if (!vocab || vocab->kind != Json::Array) return bad("missing field `vocab`");
    if (!specials || specials->kind != Json::Array) return bad("missing field `special_tokens`");
    size_t vsize = 0, nspecial = 0;
    if (!get_usize(*cfg, "default_vocab_size", &vsize, &err) ||
        !get_usize(*cfg, "default_num_special_tokens", &nspecial, &err))
        return bad(err);
    // Check every entry's fields before building anything (serde rejects the file as a whole).
    for (const Json& e : specials->arr) {
        size_t r;
        const Json* ts = e.kind == Json::Object ? e.get("token_str") : nullptr;
        const Json* ic = e.kind == Json::Object ? e.get("is_control") : nullptr;
        if (e.kind != Json::Object || !get_usize(e, "rank", &r, &err)) return bad(e.kind != Json::Object ? "special token is not an object" : err);
        if (!ts || ts->kind != Json::String) return bad("special token needs a string `token_str`");
        if (!ic || ic->kind != Json::Bool) return bad("special token needs a bool `is_control`");
    }
    for (const Json& e : vocab->arr) {
        size_t r;
        const Json* tb = e.kind == Json::Object ? e.get("token_bytes") : nullptr;
        if (e.kind != Json::Object || !get_usize(e, "rank", &r, &err)) return bad(e.kind != Json::Object ? "vocab entry is not an object" : err);
        if (!tb || tb->kind != Json::String) return bad("vocab entry needs a string `token_bytes`");
    }
    const Json* audio = root.get("audio");
    vox_tekken_audio_config ac{};
    const bool has_audio = audio && audio->kind != Json::Null;
    if (has_audio) {
        if (audio->kind != Json::Object) return bad("`audio` is not an object");
        size_t sr = 0;
        const Json* fr = audio->get("frame_rate");
        if (!get_usize(*audio, "sampling_rate", &sr, &err) ||
            !get_usize(*audio, "transcription_delay_ms", &ac.transcription_delay_ms, &err) ||
            !get_usize(*audio, "streaming_n_left_pad_tokens", &ac.streaming_n_left_pad_tokens, &err))
            return bad(err);
        if (sr > 0xFFFFFFFFull) return bad("sampling_rate out of range for u32");
        if (!fr || fr->kind != Json::Number) return bad("missing field `frame_rate`");
        ac.sampling_rate = (uint32_t)sr;
        ac.frame_rate = (float)fr->num;
    }
    // tokenizer.rs:73-76
    if (vsize == 0) return report_errorf(VOX_ERR_FORMAT, "default_vocab_size must be > 0");
    auto* t = new vox_tekken();
    t->default_vocab_size = vsize;
    t->special_token_count = nspecial;
    std::vector<int> filled(nspecial, 0);
    t->specials.resize(nspecial);
    for (const Json& e : specials->arr) {  // tokenizer.rs:78-92
        size_t rank = 0;
        get_usize(e, "rank", &rank, &err);
        if (rank >= nspecial) continue;
        const uint32_t id = (uint32_t)rank;
        const std::string& text = e.get("token_str")->str;
        t->lookup[text] = id;
        t->specials[rank] = {id, text, e.get("is_control")->b};
        filled[rank] = 1;
    }
    for (size_t r = 0; r < nspecial; ++r)  // tokenizer.rs:94-101
        if (!filled[r]) t->specials[r] = {(uint32_t)r, "<missing-special-" + std::to_string(r) + ">", true};
    t->token_bytes.resize(vsize);
    t->has_bytes.assign(vsize, 0);
    for (const Json& e : vocab->arr) {  // tokenizer.rs:103-113
        size_t rank = 0;
        get_usize(e, "rank", &rank, &err);
        const size_t id = nspecial + rank;
        if (id < nspecial || id >= vsize) continue;
        if (!b64_decode(e.get("token_bytes")->str, &t->token_bytes[id])) {
            delete t;
            return report_errorf(VOX_ERR_FORMAT, "decode base64 for vocab rank %zu", rank);
        }
        t->has_bytes[id] = 1;
    }
    t->has_audio = has_audio;
    t->audio = ac;
    *out = t;
    return VOX_OK;
}

// String::from_utf8_lossy: each maximal invalid subpart becomes one U+FFFD.
void utf8_lossy(const std::vector<uint8_t>& s, std::string* out) {
    static const char kRepl[] = "\xEF\xBF\xBD";
    size_t i = 0;
    const size_t n = s.size();
    while (i < n) {
        const uint8_t b = s[i];
        if (b < 0x80) {
            out->push_back((char)b);
            ++i;
            continue;
        }
        int len;
        uint8_t lo = 0x80, hi = 0xBF;  // range of the second byte
        if (b >= 0xC2 && b <= 0xDF) len = 2;
        else if (b == 0xE0) { len = 3; lo = 0xA0; }
        else if ((b >= 0xE1 && b <= 0xEC) || b == 0xEE || b == 0xEF) len = 3;
        else if (b == 0xED) { len = 3; hi = 0x9F; }
        else if (b == 0xF0) { len = 4; lo = 0x90; }
        else if (b >= 0xF1 && b <= 0xF3) len = 4;
        else if (b == 0xF4) { len = 4; hi = 0x8F; }
        else {
            out->append(kRepl);
            ++i;
            continue;
        }
        int k = 1;
        for (; k < len; ++k) {
            if (i + k >= n) break;
            const uint8_t c = s[i + k];
            const uint8_t l = k == 1 ? lo : 0x80, h = k == 1 ? hi : 0xBF;
            if (c < l || c > h) break;
        }
        if (k == len) {
            out->append(reinterpret_cast<const char*>(&s[i]), len);
            i += len;
        } else {
            out->append(kRepl);
            i += k;
        }
    }
}

}  // namespace

extern "C" int vox_tekken_from_json(const char* json, size_t len, vox_tekken** out) {
    if (!json || !out) return report_errorf(VOX_ERR_INVALID_ARG, "null json or output");
    *out = nullptr;
    return parse(json, len, out);
}

extern "C" int vox_tekken_from_path(const char* path, vox_tekken** out) {
    if (!path || !out) return report_errorf(VOX_ERR_INVALID_ARG, "null path or output");
    *out = nullptr;
    std::ifstream f(path, std::ios::binary);
    if (!f) return report_errorf(VOX_ERR_IO, "read %s", path);
    std::stringstream ss;
    ss << f.rdbuf();
    const std::string text = ss.str();
    return parse(text.data(), text.size(), out);
}

extern "C" void vox_tekken_destroy(vox_tekken* t) { delete t; }

extern "C" size_t vox_tekken_default_vocab_size(const vox_tekken* t) { return t ? t->default_vocab_size : 0; }
extern "C" size_t vox_tekken_special_token_count(const vox_tekken* t) { return t ? t->special_token_count : 0; }

extern "C" int vox_tekken_special_id(const vox_tekken* t, const char* text, uint32_t* id) {
    if (!t || !text) return 0;
    auto it = t->lookup.find(text);
    if (it == t->lookup.end()) return 0;
    if (id) *id = it->second;
    return 1;
}

extern "C" int vox_tekken_audio(const vox_tekken* t, vox_tekken_audio_config* out) {
    if (!t || !t->has_audio) return 0;
    if (out) *out = t->audio;
    return 1;
}

extern "C" int vox_tekken_transcription_delay_tokens(const vox_tekken* t, size_t* out) {
    if (!t || !t->has_audio) return 0;
    // tokenizer.rs:167-171: f32 seconds * frame rate, rounded half away from
    // zero, then `as usize` (negative and NaN saturate to 0).
    const float seconds = (float)t->audio.transcription_delay_ms / 1000.0f;
    const float r = std::round(seconds * t->audio.frame_rate);
    size_t v = 0;
    if (r > 0.0f) v = r >= 1.8446744e19f ? SIZE_MAX : (size_t)r;
    if (out) *out = v;
    return 1;
}

extern "C" int vox_tekken_default_prompt_ids(const vox_tekken* t, uint32_t* out, size_t cap, size_t* len) {
    uint32_t bos, pad;
    size_t delay;
    // tokenizer.rs:171-184: None unless bos, pad, audio and the delay exist.
    if (!vox_tekken_special_id(t, "<s>", &bos) || !vox_tekken_special_id(t, "[STREAMING_PAD]", &pad) ||
        !t->has_audio || !vox_tekken_transcription_delay_tokens(t, &delay))
        return 0;
    const size_t n = 1 + t->audio.streaming_n_left_pad_tokens + delay;
    for (size_t i = 0; out && i < n && i < cap; ++i) out[i] = i == 0 ? bos : pad;
    if (len) *len = n;
    return 1;
}

extern "C" int vox_tekken_decode_token_bytes(const vox_tekken* t, uint32_t token_id, const uint8_t** bytes,
                                             size_t* len) {
    if (!t) return 0;
    const size_t idx = token_id;  // tokenizer.rs:186-203
    if (idx >= t->default_vocab_size) return 0;
    if (idx < t->special_token_count) {
        const auto& st = t->specials[idx];
        if (st.is_control) return 0;
        if (bytes) *bytes = reinterpret_cast<const uint8_t*>(st.text.data());
        if (len) *len = st.text.size();
        return 1;
    }
    if (!t->has_bytes[idx]) return 0;
    if (bytes) *bytes = t->token_bytes[idx].data();
    if (len) *len = t->token_bytes[idx].size();
    return 1;
}

extern "C" size_t vox_tekken_decode_to_utf8_lossy(const vox_tekken* t, const uint32_t* ids, size_t n, char* out,
                                                  size_t cap) {
    if (!t || (!ids && n)) return 0;
    std::vector<uint8_t> raw;  // tokenizer.rs:204-213
    for (size_t i = 0; i < n; ++i) {
        const uint8_t* b;
        size_t l;
        if (vox_tekken_decode_token_bytes(t, ids[i], &b, &l)) raw.insert(raw.end(), b, b + l);
    }
    std::string s;
    utf8_lossy(raw, &s);
    if (out && cap) {
        const size_t k = s.size() < cap - 1 ? s.size() : cap - 1;
        std::memcpy(out, s.data(), k);
        out[k] = '\0';
    }
    return s.size();
}
