// Host-side file formats: a small JSON value type and parser (manifest.json, run.json),
// SHA-256 (FIPS 180-4; the package digest check of weights.rs:29-40), a strict F32
// safetensors reader (weights.rs:42-144) and WAV read / write (the float32 writer of
// crates/ancha-audio/src/lib.rs:51-67).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

namespace ancha {

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json* find(const std::string& key) const;
    const Json& at(const std::string& key) const;  // throws if missing
    int64_t as_int() const;
    int as_int32() const;  // throws outside the int range
    double as_double() const;
    bool as_bool() const;
    const std::string& as_string() const;

    static Json parse(const std::string& text);  // throws std::runtime_error
    std::string dump(int indent = 2) const;
    static Json make_object() { Json j; j.kind = Object; return j; }
    static Json make_array() { Json j; j.kind = Array; return j; }
    static Json of(double v) { Json j; j.kind = Number; j.num = v; return j; }
    static Json of(const std::string& v) { Json j; j.kind = String; j.str = v; return j; }
    static Json of_bool(bool v) { Json j; j.kind = Bool; j.b = v; return j; }
    void set(const std::string& key, Json v);
};

std::string sha256_hex(const uint8_t* data, size_t size);

std::string read_file(const std::string& path);  // throws std::runtime_error

// Strict F32 safetensors: every tensor must be F32, shapes are checked on take(), and
// finish() rejects tensors that were never taken.
class SafeTensors {
public:
    explicit SafeTensors(const std::string& bytes);
    std::vector<float> take(const std::string& name, const std::vector<int64_t>& shape);
    size_t finish() const;  // number of tensors used; throws on unused tensors
    bool has(const std::string& name) const { return index_.count(name) != 0; }

private:
    struct Entry { std::vector<int64_t> shape; size_t begin, end; std::string dtype; };
    const std::string& bytes_;
    size_t data_offset_ = 0;
    std::map<std::string, Entry> index_;
    std::set<std::string> used_;
};

struct Audio {
    int sample_rate = 0;
    std::vector<std::vector<float>> planes;
    int64_t samples() const { return planes.empty() ? 0 : (int64_t)planes[0].size(); }
};

Audio read_wav(const std::string& path);                       // PCM16/24/32 or float32
void write_wav(const std::string& path, const Audio& audio);   // float32

}  // namespace ancha
