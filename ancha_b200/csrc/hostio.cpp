// Host-side file formats (see hostio.hpp).
#include "hostio.hpp"

#include <climits>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>

namespace ancha {

// ---------------------------------------------------------------------------------------
// JSON
// ---------------------------------------------------------------------------------------
const Json* Json::find(const std::string& key) const {
    if (kind != Object) return nullptr;
    for (auto& kv : obj)
        if (kv.first == key) return &kv.second;
    return nullptr;
}
const Json& Json::at(const std::string& key) const {
    const Json* j = find(key);
    if (!j) throw std::runtime_error("missing key '" + key + "'");
    return *j;
}
int64_t Json::as_int() const {
    // Integers beyond 2^53 are not exact in a double (and beyond 2^63 have no int64 value).
    if (kind != Number || std::floor(num) != num || std::fabs(num) > 9007199254740992.0)
        throw std::runtime_error("expected an integer");
    return (int64_t)num;
}
int Json::as_int32() const {
    const int64_t v = as_int();
    if (v < INT32_MIN || v > INT32_MAX) throw std::runtime_error("integer out of range");
    return (int)v;
}
double Json::as_double() const {
    if (kind != Number) throw std::runtime_error("expected a number");
    return num;
}
bool Json::as_bool() const {
    if (kind != Bool) throw std::runtime_error("expected a boolean");
    return b;
}
const std::string& Json::as_string() const {
    if (kind != String) throw std::runtime_error("expected a string");
    return str;
}
void Json::set(const std::string& key, Json v) {
    for (auto& kv : obj)
        if (kv.first == key) { kv.second = std::move(v); return; }
    obj.emplace_back(key, std::move(v));
}

namespace {
struct Parser {
    static constexpr int kMaxDepth = 256;  // nesting of arrays / objects; bounds the recursion
    const std::string& s;
    size_t i = 0;
    int depth = 0;
    void ws() { while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i; }
    [[noreturn]] void err(const char* what) {
        throw std::runtime_error(std::string("JSON: ") + what + " at offset " + std::to_string(i));
    }
    char peek() { ws(); if (i >= s.size()) err("unexpected end"); return s[i]; }
    void expect(char c) { if (peek() != c) err("unexpected character"); ++i; }
    std::string string() {
        expect('"');
        std::string out;
        while (true) {
            if (i >= s.size()) err("unterminated string");
            char c = s[i++];
            if (c == '"') break;
            if (c != '\\') { out.push_back(c); continue; }
            if (i >= s.size()) err("bad escape");
            char e = s[i++];
            switch (e) {
                case '"': out.push_back('"'); break;
                case '\\': out.push_back('\\'); break;
                case '/': out.push_back('/'); break;
                case 'b': out.push_back('\b'); break;
                case 'f': out.push_back('\f'); break;
                case 'n': out.push_back('\n'); break;
                case 'r': out.push_back('\r'); break;
                case 't': out.push_back('\t'); break;
                case 'u': {
                    if (i + 4 > s.size()) err("bad unicode escape");
                    unsigned cp = 0;
                    for (int k = 0; k < 4; ++k) {
                        const char h = s[i + k];
                        const int v = h >= '0' && h <= '9' ? h - '0' : h >= 'a' && h <= 'f' ? h - 'a' + 10
                                    : h >= 'A' && h <= 'F' ? h - 'A' + 10 : -1;
                        if (v < 0) err("bad unicode escape");
                        cp = cp << 4 | (unsigned)v;
                    }
                    i += 4;
                    if (cp < 0x80) out.push_back((char)cp);
                    else if (cp < 0x800) { out.push_back((char)(0xC0 | (cp >> 6))); out.push_back((char)(0x80 | (cp & 0x3F))); }
                    else { out.push_back((char)(0xE0 | (cp >> 12))); out.push_back((char)(0x80 | ((cp >> 6) & 0x3F))); out.push_back((char)(0x80 | (cp & 0x3F))); }
                    break;
                }
                default: err("bad escape");
            }
        }
        return out;
    }
    Json value() {
        char c = peek();
        Json j;
        if ((c == '{' || c == '[') && depth >= kMaxDepth) err("nesting too deep");
        struct Level { int& d; explicit Level(int& d_) : d(d_) { ++d; } ~Level() { --d; } } level(depth);
        if (c == '{') {
            ++i; j.kind = Json::Object;
            if (peek() == '}') { ++i; return j; }
            while (true) {
                std::string k = string();
                expect(':');
                for (auto& kv : j.obj) if (kv.first == k) err("duplicate key");
                j.obj.emplace_back(k, value());
                char d = peek(); ++i;
                if (d == '}') break;
                if (d != ',') err("expected , or }");
            }
        } else if (c == '[') {
            ++i; j.kind = Json::Array;
            if (peek() == ']') { ++i; return j; }
            while (true) {
                j.arr.push_back(value());
                char d = peek(); ++i;
                if (d == ']') break;
                if (d != ',') err("expected , or ]");
            }
        } else if (c == '"') {
            j.kind = Json::String; j.str = string();
        } else if (s.compare(i, 4, "true") == 0) { i += 4; j.kind = Json::Bool; j.b = true; }
        else if (s.compare(i, 5, "false") == 0) { i += 5; j.kind = Json::Bool; j.b = false; }
        else if (s.compare(i, 4, "null") == 0) { i += 4; j.kind = Json::Null; }
        else {
            const char* b = s.c_str() + i;
            char* e = nullptr;
            double v = std::strtod(b, &e);
            if (e == b) err("bad value");
            i += (size_t)(e - b);
            j.kind = Json::Number; j.num = v;
        }
        return j;
    }
};

void dump_string(std::ostringstream& o, const std::string& s) {
    o << '"';
    for (unsigned char c : s) {
        switch (c) {
            case '"': o << "\\\""; break;
            case '\\': o << "\\\\"; break;
            case '\n': o << "\\n"; break;
            case '\r': o << "\\r"; break;
            case '\t': o << "\\t"; break;
            default:
                if (c < 0x20) { char buf[8]; std::snprintf(buf, sizeof buf, "\\u%04x", c); o << buf; }
                else o << (char)c;
        }
    }
    o << '"';
}

void dump_value(std::ostringstream& o, const Json& j, int indent, int depth) {
    auto nl = [&](int d) { if (indent > 0) { o << '\n'; for (int k = 0; k < d * indent; ++k) o << ' '; } };
    switch (j.kind) {
        case Json::Null: o << "null"; break;
        case Json::Bool: o << (j.b ? "true" : "false"); break;
        case Json::Number: {
            if (!std::isfinite(j.num)) { o << "null"; break; }
            if (std::floor(j.num) == j.num && std::fabs(j.num) < 9e15) { o << (int64_t)j.num; break; }
            char buf[40]; std::snprintf(buf, sizeof buf, "%.17g", j.num); o << buf; break;
        }
        case Json::String: dump_string(o, j.str); break;
        case Json::Array: {
            o << '[';
            bool scalar = true;
            for (auto& v : j.arr) if (v.kind == Json::Array || v.kind == Json::Object) scalar = false;
            for (size_t k = 0; k < j.arr.size(); ++k) {
                if (k) o << ',';
                if (!scalar) nl(depth + 1); else if (k && indent) o << ' ';
                dump_value(o, j.arr[k], indent, depth + 1);
            }
            if (!scalar && !j.arr.empty()) nl(depth);
            o << ']';
            break;
        }
        case Json::Object: {
            o << '{';
            for (size_t k = 0; k < j.obj.size(); ++k) {
                if (k) o << ',';
                nl(depth + 1);
                dump_string(o, j.obj[k].first);
                o << (indent ? ": " : ":");
                dump_value(o, j.obj[k].second, indent, depth + 1);
            }
            if (!j.obj.empty()) nl(depth);
            o << '}';
            break;
        }
    }
}
}  // namespace

Json Json::parse(const std::string& text) {
    Parser p{text};
    Json j = p.value();
    p.ws();
    if (p.i != text.size()) p.err("trailing characters");
    return j;
}

std::string Json::dump(int indent) const {
    std::ostringstream o;
    dump_value(o, *this, indent, 0);
    return o.str();
}

// ---------------------------------------------------------------------------------------
// SHA-256 (FIPS 180-4). The round constants K and the initial hash H0 are the first 32
// fractional bits of the cube / square roots of the first primes, computed here exactly
// with 128-bit integer roots.
// ---------------------------------------------------------------------------------------
namespace {
uint64_t iroot(unsigned __int128 n, int k) {  // floor(n^(1/k)), k = 2 or 3
    uint64_t lo = 0, hi = (uint64_t)1 << 40;
    while (lo < hi) {
        uint64_t mid = lo + (hi - lo + 1) / 2;
        unsigned __int128 p = (unsigned __int128)mid * mid;
        if (k == 3) p *= mid;
        if (p <= n) lo = mid; else hi = mid - 1;
    }
    return lo;
}
struct ShaConstants {
    uint32_t k[64], h0[8];
    ShaConstants() {
        int primes[64], n = 0;
        for (int c = 2; n < 64; ++c) {
            bool prime = true;
            for (int d = 2; d * d <= c; ++d) if (c % d == 0) { prime = false; break; }
            if (prime) primes[n++] = c;
        }
        for (int i = 0; i < 64; ++i)
            k[i] = (uint32_t)iroot((unsigned __int128)primes[i] << 96, 3);
        for (int i = 0; i < 8; ++i)
            h0[i] = (uint32_t)iroot((unsigned __int128)primes[i] << 64, 2);
    }
};
const ShaConstants& sha_constants() { static ShaConstants c; return c; }
inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void sha_block(uint32_t h[8], const uint8_t* p, const uint32_t* K) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
        w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
        uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
        uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
        uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
        uint32_t ch = (e & f) ^ (~e & g);
        uint32_t t1 = hh + S1 + ch + K[i] + w[i];
        uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
        uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
        uint32_t t2 = S0 + mj;
        hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}
}  // namespace

std::string sha256_hex(const uint8_t* data, size_t size) {
    const ShaConstants& C = sha_constants();
    uint32_t h[8];
    std::memcpy(h, C.h0, sizeof h);
    size_t full = size / 64;
    for (size_t b = 0; b < full; ++b) sha_block(h, data + 64 * b, C.k);
    uint8_t tail[128] = {0};
    size_t rem = size - 64 * full;
    std::memcpy(tail, data + 64 * full, rem);
    tail[rem] = 0x80;
    size_t tlen = rem + 1 + 8 <= 64 ? 64 : 128;
    uint64_t bits = (uint64_t)size * 8;
    for (int i = 0; i < 8; ++i) tail[tlen - 1 - i] = (uint8_t)(bits >> (8 * i));
    for (size_t b = 0; b < tlen; b += 64) sha_block(h, tail + b, C.k);
    char out[65];
    for (int i = 0; i < 8; ++i) std::snprintf(out + 8 * i, 9, "%08x", h[i]);
    return std::string(out, 64);
}

std::string read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("read " + path);
    std::ostringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

// ---------------------------------------------------------------------------------------
// safetensors
// ---------------------------------------------------------------------------------------
SafeTensors::SafeTensors(const std::string& bytes) : bytes_(bytes) {
    if (bytes.size() < 8) throw std::runtime_error("safetensors: file too small");
    uint64_t n = 0;
    for (int i = 0; i < 8; ++i) n |= (uint64_t)(uint8_t)bytes[i] << (8 * i);
    if (n > bytes.size() - 8) throw std::runtime_error("safetensors: bad header length");
    Json header = Json::parse(bytes.substr(8, n));
    data_offset_ = 8 + n;
    if (header.kind != Json::Object) throw std::runtime_error("safetensors: bad header");
    for (auto& kv : header.obj) {
        if (kv.first == "__metadata__") continue;
        Entry e;
        e.dtype = kv.second.at("dtype").as_string();
        for (auto& d : kv.second.at("shape").arr) {
            e.shape.push_back(d.as_int());
            if (e.shape.back() < 0) throw std::runtime_error("safetensors: negative dimension: " + kv.first);
        }
        auto& off = kv.second.at("data_offsets").arr;
        if (off.size() != 2) throw std::runtime_error("safetensors: bad offsets");
        const int64_t begin = off[0].as_int(), end = off[1].as_int();
        // Offsets are relative to the data section; compare without forming a sum that could wrap.
        if (begin < 0 || end < begin || (uint64_t)end > bytes.size() - data_offset_)
            throw std::runtime_error("safetensors: tensor out of range: " + kv.first);
        e.begin = (size_t)begin;
        e.end = (size_t)end;
        index_[kv.first] = e;
    }
}

std::vector<float> SafeTensors::take(const std::string& name, const std::vector<int64_t>& shape) {
    auto it = index_.find(name);
    if (it == index_.end()) throw std::runtime_error("missing tensor " + name);
    const Entry& e = it->second;
    if (e.shape != shape) {
        std::string got, want;
        for (auto d : e.shape) got += std::to_string(d) + ",";
        for (auto d : shape) want += std::to_string(d) + ",";
        throw std::runtime_error(name + ": expected [" + want + "], got [" + got + "]");
    }
    if (e.dtype != "F32") throw std::runtime_error(name + ": schema 1 requires F32 weights, got " + e.dtype);
    size_t count = 1;  // bounded by the tensor's byte range, so count · 4 cannot wrap
    for (auto d : shape) {
        if (d < 0 || (d && count > (e.end - e.begin) / 4 / (size_t)d)) throw std::runtime_error(name + ": byte size mismatch");
        count *= (size_t)d;
    }
    if (e.end - e.begin != count * 4) throw std::runtime_error(name + ": byte size mismatch");
    std::vector<float> out(count);
    std::memcpy(out.data(), bytes_.data() + data_offset_ + e.begin, count * 4);
    for (float v : out)
        if (!std::isfinite(v)) throw std::runtime_error(name + ": non-finite weight");
    used_.insert(name);
    return out;
}

size_t SafeTensors::finish() const {
    std::string unused;
    int n = 0;
    for (auto& kv : index_)
        if (!used_.count(kv.first) && n < 8) { unused += kv.first + " "; ++n; }
    if (n) throw std::runtime_error("unrecognized checkpoint tensors: " + unused);
    return used_.size();
}

// ---------------------------------------------------------------------------------------
// WAV
// ---------------------------------------------------------------------------------------
namespace {
uint32_t le32(const uint8_t* p) { return p[0] | p[1] << 8 | p[2] << 16 | (uint32_t)p[3] << 24; }
uint16_t le16(const uint8_t* p) { return (uint16_t)(p[0] | p[1] << 8); }
void put32(std::string& s, uint32_t v) { for (int i = 0; i < 4; ++i) s.push_back((char)(v >> (8 * i))); }
void put16(std::string& s, uint16_t v) { s.push_back((char)v); s.push_back((char)(v >> 8)); }
}  // namespace

Audio read_wav(const std::string& path) {
    std::string raw = read_file(path);
    const uint8_t* p = reinterpret_cast<const uint8_t*>(raw.data());
    if (raw.size() < 12 || std::memcmp(p, "RIFF", 4) || std::memcmp(p + 8, "WAVE", 4))
        throw std::runtime_error(path + ": not a RIFF/WAVE file");
    size_t pos = 12;
    int format = -1, channels = 0, bits = 0;
    uint32_t rate = 0;
    const uint8_t* data = nullptr;
    size_t data_size = 0;
    while (pos + 8 <= raw.size()) {
        uint32_t size = le32(p + pos + 4);
        const uint8_t* body = p + pos + 8;
        if (pos + 8 + size > raw.size()) size = (uint32_t)(raw.size() - pos - 8);
        if (!std::memcmp(p + pos, "fmt ", 4) && size >= 16) {
            format = le16(body);
            channels = le16(body + 2);
            rate = le32(body + 4);
            bits = le16(body + 14);
            if (format == 0xFFFE && size >= 26) format = le16(body + 24);
        } else if (!std::memcmp(p + pos, "data", 4)) {
            data = body;
            data_size = size;
        }
        pos += 8 + size + (size & 1);
    }
    if (!data || format < 0) throw std::runtime_error(path + ": missing fmt or data chunk");
    if (channels < 1 || channels > 2) throw std::runtime_error(path + ": only mono or stereo WAV is supported");
    const int bytes = bits / 8;
    if (!((format == 1 && (bits == 16 || bits == 24 || bits == 32)) || (format == 3 && bits == 32)))
        throw std::runtime_error(path + ": unsupported WAV encoding");
    const size_t frames = data_size / (size_t)(bytes * channels);
    Audio a;
    a.sample_rate = (int)rate;
    a.planes.assign(channels, std::vector<float>(frames));
    for (size_t f = 0; f < frames; ++f)
        for (int c = 0; c < channels; ++c) {
            const uint8_t* s = data + (f * channels + c) * bytes;
            float v;
            if (format == 3) std::memcpy(&v, s, 4);
            else if (bits == 16) v = (float)(int16_t)le16(s) / 32768.f;
            else if (bits == 24) v = (float)((int32_t)((uint32_t)s[0] << 8 | (uint32_t)s[1] << 16 | (uint32_t)s[2] << 24) >> 8) / 8388608.f;
            else v = (float)((double)(int32_t)le32(s) / 2147483648.0);
            a.planes[c][f] = v;
        }
    return a;
}

void write_wav(const std::string& path, const Audio& audio) {
    const int channels = (int)audio.planes.size();
    const int64_t n = audio.samples();
    if (channels == 0 || n == 0) throw std::runtime_error("write_wav: empty audio");
    std::string s;
    // RIFF sizes are 32-bit: refuse what does not fit, as the reference's WAV writer does.
    if ((uint64_t)n * channels * 4 > 0xFFFFFFFFull - 36) throw std::runtime_error("write_wav: more than 4 GiB of samples");
    const uint32_t data_bytes = (uint32_t)(n * channels * 4);
    s.append("RIFF");
    put32(s, 36 + data_bytes);
    s.append("WAVEfmt ");
    put32(s, 16);
    put16(s, 3);
    put16(s, (uint16_t)channels);
    put32(s, (uint32_t)audio.sample_rate);
    put32(s, (uint32_t)audio.sample_rate * channels * 4);
    put16(s, (uint16_t)(channels * 4));
    put16(s, 32);
    s.append("data");
    put32(s, data_bytes);
    s.reserve(s.size() + data_bytes);
    for (int64_t i = 0; i < n; ++i)
        for (int c = 0; c < channels; ++c) {
            float v = audio.planes[c][i];
            s.append(reinterpret_cast<const char*>(&v), 4);
        }
    std::ofstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("write " + path);
    f.write(s.data(), (std::streamsize)s.size());
    if (!f) throw std::runtime_error("write " + path);
}

}  // namespace ancha
