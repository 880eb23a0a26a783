// Host-side support for the packed checkpoint format: JSON, SHA-256 and the manifest written by
// the reference's export_packed.rs:13-103 ({"schema_version":1, "scheme":"q4-w4a8-e4-r4-g64",
// "group_size":64, "layers":[{"file","bytes","tensors":[{"name","shape","start","end"}]}],
// "embedding", "readout", "norm", "files":{name:{"bytes","sha256"}}, ...}).
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>

#include "packed_io.h"

namespace dbio {

const Json* Json::get(const std::string& key) const {
    if (kind != OBJ) return nullptr;
    for (const auto& kv : obj)
        if (kv.first == key) return &kv.second;
    return nullptr;
}

namespace {

struct Parser {
    const std::string& s;
    size_t i = 0;
    std::string err;
    explicit Parser(const std::string& text) : s(text) {}
    void ws() {
        while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
    }
    bool fail(const char* what) {
        if (err.empty()) err = std::string(what) + " at byte " + std::to_string(i);
        return false;
    }
    bool lit(const char* w) {
        const size_t n = std::strlen(w);
        if (s.compare(i, n, w) != 0) return fail("bad literal");
        i += n;
        return true;
    }
    static void utf8(uint32_t c, std::string* out) {
        if (c < 0x80) {
            out->push_back((char)c);
        } else if (c < 0x800) {
            out->push_back((char)(0xC0 | (c >> 6)));
            out->push_back((char)(0x80 | (c & 0x3F)));
        } else if (c < 0x10000) {
            out->push_back((char)(0xE0 | (c >> 12)));
            out->push_back((char)(0x80 | ((c >> 6) & 0x3F)));
            out->push_back((char)(0x80 | (c & 0x3F)));
        } else {
            out->push_back((char)(0xF0 | (c >> 18)));
            out->push_back((char)(0x80 | ((c >> 12) & 0x3F)));
            out->push_back((char)(0x80 | ((c >> 6) & 0x3F)));
            out->push_back((char)(0x80 | (c & 0x3F)));
        }
    }
    bool hex4(uint32_t* v) {
        if (i + 4 > s.size()) return fail("short escape");
        *v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = s[i++];
            *v <<= 4;
            if (c >= '0' && c <= '9') *v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') *v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') *v |= (uint32_t)(c - 'A' + 10);
            else return fail("bad escape");
        }
        return true;
    }
    bool string(std::string* out) {
        if (i >= s.size() || s[i] != '"') return fail("expected string");
        ++i;
        while (i < s.size() && s[i] != '"') {
            if (s[i] != '\\') {
                out->push_back(s[i++]);
                continue;
            }
            if (++i >= s.size()) return fail("short escape");
            const char e = s[i++];
            switch (e) {
                case '"': out->push_back('"'); break;
                case '\\': out->push_back('\\'); break;
                case '/': out->push_back('/'); break;
                case 'b': out->push_back('\b'); break;
                case 'f': out->push_back('\f'); break;
                case 'n': out->push_back('\n'); break;
                case 'r': out->push_back('\r'); break;
                case 't': out->push_back('\t'); break;
                case 'u': {
                    uint32_t c = 0;
                    if (!hex4(&c)) return false;
                    if (c >= 0xD800 && c < 0xDC00 && i + 6 <= s.size() && s[i] == '\\' && s[i + 1] == 'u') {
                        i += 2;
                        uint32_t lo = 0;
                        if (!hex4(&lo)) return false;
                        c = 0x10000 + ((c - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(c, out);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (i >= s.size()) return fail("unterminated string");
        ++i;
        return true;
    }
    bool value(Json* v, int depth) {
        if (depth > 64) return fail("nesting too deep");
        ws();
        if (i >= s.size()) return fail("unexpected end");
        const char c = s[i];
        if (c == '{') {
            v->kind = Json::OBJ;
            ++i;
            ws();
            if (i < s.size() && s[i] == '}') return ++i, true;
            for (;;) {
                ws();
                std::string key;
                if (!string(&key)) return false;
                ws();
                if (i >= s.size() || s[i] != ':') return fail("expected ':'");
                ++i;
                Json child;
                if (!value(&child, depth + 1)) return false;
                v->obj.emplace_back(std::move(key), std::move(child));
                ws();
                if (i < s.size() && s[i] == ',') { ++i; continue; }
                if (i < s.size() && s[i] == '}') return ++i, true;
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v->kind = Json::ARR;
            ++i;
            ws();
            if (i < s.size() && s[i] == ']') return ++i, true;
            for (;;) {
                Json child;
                if (!value(&child, depth + 1)) return false;
                v->arr.push_back(std::move(child));
                ws();
                if (i < s.size() && s[i] == ',') { ++i; continue; }
                if (i < s.size() && s[i] == ']') return ++i, true;
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v->kind = Json::STR;
            return string(&v->str);
        }
        if (c == 't') { v->kind = Json::BOOL; v->b = true; return lit("true"); }
        if (c == 'f') { v->kind = Json::BOOL; v->b = false; return lit("false"); }
        if (c == 'n') { v->kind = Json::NUL; return lit("null"); }
        const size_t start = i;
        if (s[i] == '-') ++i;
        while (i < s.size() && (isdigit((unsigned char)s[i]) || s[i] == '.' || s[i] == 'e' || s[i] == 'E' ||
                                s[i] == '+' || s[i] == '-'))
            ++i;
        if (i == start) return fail("unexpected character");
        v->kind = Json::NUM;
        v->num = std::strtod(s.c_str() + start, nullptr);
        return true;
    }
};

// ---- SHA-256, FIPS 180-4 section 6.2
const uint32_t K256[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5, 0xd807aa98,
    0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786,
    0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8,
    0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13,
    0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85, 0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819,
    0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a,
    0x5b9cca4f, 0x682e6ff3, 0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7,
    0xc67178f2};
inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
void sha256_block(uint32_t* h, const uint8_t* p) {
    uint32_t w[64];
    for (int t = 0; t < 16; ++t)
        w[t] = (uint32_t)p[4 * t] << 24 | (uint32_t)p[4 * t + 1] << 16 | (uint32_t)p[4 * t + 2] << 8 | p[4 * t + 3];
    for (int t = 16; t < 64; ++t) {
        const uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
        const uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
        w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int t = 0; t < 64; ++t) {
        const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + K256[t] + w[t];
        const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
        hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

bool num_u64(const Json* j, uint64_t* out) {
    if (!j || j->kind != Json::NUM || j->num < 0) return false;
    *out = (uint64_t)j->num;
    return true;
}
std::string str_or_empty(const Json* j) { return j && j->kind == Json::STR ? j->str : std::string(); }

}  // namespace

bool json_parse(const std::string& text, Json* out, std::string* err) {
    Parser p(text);
    if (!p.value(out, 0)) {
        if (err) *err = p.err;
        return false;
    }
    p.ws();
    if (p.i != text.size()) {
        if (err) *err = "trailing characters at byte " + std::to_string(p.i);
        return false;
    }
    return true;
}

std::string json_quote(const std::string& s) {
    std::string o = "\"";
    for (char c : s) {
        if (c == '"' || c == '\\') { o.push_back('\\'); o.push_back(c); }
        else if ((unsigned char)c < 0x20) {
            char b[8];
            std::snprintf(b, sizeof b, "\\u%04x", (unsigned)(unsigned char)c);
            o += b;
        } else {
            o.push_back(c);
        }
    }
    return o + "\"";
}

std::string sha256_hex(const uint8_t* data, size_t n) {
    uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    size_t full = n / 64;
    for (size_t b = 0; b < full; ++b) sha256_block(h, data + 64 * b);
    uint8_t tail[128] = {};
    const size_t rem = n - 64 * full;
    std::memcpy(tail, data + 64 * full, rem);
    tail[rem] = 0x80;
    const size_t tail_len = rem + 9 <= 64 ? 64 : 128;
    const uint64_t bits = (uint64_t)n * 8;
    for (int k = 0; k < 8; ++k) tail[tail_len - 1 - k] = (uint8_t)(bits >> (8 * k));
    for (size_t b = 0; b < tail_len / 64; ++b) sha256_block(h, tail + 64 * b);
    char hex[65];
    for (int k = 0; k < 8; ++k) std::snprintf(hex + 8 * k, 9, "%08x", h[k]);
    return std::string(hex, 64);
}

const TensorEntry* LayerEntry::find_suffix(const std::string& suffix) const {
    for (const auto& t : tensors)
        if (t.name.size() >= suffix.size() && t.name.compare(t.name.size() - suffix.size(), suffix.size(), suffix) == 0)
            return &t;
    return nullptr;
}

bool read_manifest(const std::string& path, Manifest* m, std::string* err) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return *err = "cannot open manifest " + path, false;
    std::stringstream ss;
    ss << f.rdbuf();
    Json j;
    if (!json_parse(ss.str(), &j, err)) return *err = "manifest: " + *err, false;
    if (j.kind != Json::OBJ) return *err = "manifest is not an object", false;
    uint64_t v = 0;
    if (!num_u64(j.get("schema_version"), &v) || v != 1) return *err = "unsupported schema_version", false;
    m->schema_version = 1;
    m->revision = str_or_empty(j.get("revision"));
    m->scheme = str_or_empty(j.get("scheme"));
    if (!num_u64(j.get("group_size"), &v) || v != 64) return *err = "group_size must be 64", false;
    m->group_size = 64;
    if (m->scheme.rfind("q4-", 0) == 0) m->bits = 4;
    else if (m->scheme.rfind("q8-", 0) == 0) m->bits = 8;
    else return *err = "unknown scheme " + m->scheme, false;
    num_u64(j.get("group_bytes"), &m->group_bytes);
    num_u64(j.get("embedding_row_bytes"), &m->embedding_row_bytes);
    num_u64(j.get("decoder_bytes"), &m->decoder_bytes);
    m->embedding = str_or_empty(j.get("embedding"));
    m->readout = str_or_empty(j.get("readout"));
    m->norm = str_or_empty(j.get("norm"));
    const Json* layers = j.get("layers");
    if (!layers || layers->kind != Json::ARR) return *err = "manifest has no layers", false;
    for (const Json& l : layers->arr) {
        LayerEntry e;
        e.file = str_or_empty(l.get("file"));
        num_u64(l.get("bytes"), &e.bytes);
        const Json* ts = l.get("tensors");
        if (e.file.empty() || !ts || ts->kind != Json::ARR) return *err = "malformed layer entry", false;
        for (const Json& t : ts->arr) {
            TensorEntry te;
            te.name = str_or_empty(t.get("name"));
            const Json* sh = t.get("shape");
            if (te.name.empty() || !sh || sh->kind != Json::ARR || !num_u64(t.get("start"), &te.start) ||
                !num_u64(t.get("end"), &te.end) || te.end < te.start || te.end > e.bytes)
                return *err = "malformed tensor entry in " + e.file, false;
            for (const Json& d : sh->arr) {
                if (d.kind != Json::NUM || d.num < 0) return *err = "malformed shape of " + te.name, false;
                te.shape.push_back((int64_t)d.num);
            }
            e.tensors.push_back(std::move(te));
        }
        m->layers.push_back(std::move(e));
    }
    const Json* files = j.get("files");
    if (!files || files->kind != Json::OBJ) return *err = "manifest has no files", false;
    for (const auto& kv : files->obj) {
        uint64_t bytes = 0;
        num_u64(kv.second.get("bytes"), &bytes);
        m->files[kv.first] = {bytes, str_or_empty(kv.second.get("sha256"))};
    }
    return true;
}

bool read_checked(const std::string& dir, const std::string& name, const Manifest& m, bool verify,
                  std::vector<uint8_t>* out, std::string* err) {
    if (name.empty() || name.find('/') != std::string::npos || name.find('\\') != std::string::npos || name == "..")
        return *err = "invalid file name in manifest: " + name, false;
    auto it = m.files.find(name);
    if (it == m.files.end()) return *err = "file not listed in manifest: " + name, false;
    std::ifstream f(dir + "/" + name, std::ios::binary | std::ios::ate);
    if (!f) return *err = "cannot open " + name, false;
    const std::streamoff size = f.tellg();
    if (size < 0 || (uint64_t)size != it->second.first)
        return *err = name + ": size " + std::to_string((long long)size) + " != manifest " +
                      std::to_string((unsigned long long)it->second.first), false;
    out->resize((size_t)size);
    f.seekg(0);
    if (size > 0 && !f.read(reinterpret_cast<char*>(out->data()), size)) return *err = "cannot read " + name, false;
    if (verify && sha256_hex(out->data(), out->size()) != it->second.second)
        return *err = name + ": sha256 does not match the manifest", false;
    return true;
}

bool write_file(const std::string& path, const void* data, size_t n, std::string* err) {
    std::ofstream f(path, std::ios::binary | std::ios::trunc);
    if (!f || (n && !f.write(static_cast<const char*>(data), (std::streamsize)n)))
        return *err = "cannot write " + path, false;
    return true;
}

}  // namespace dbio
