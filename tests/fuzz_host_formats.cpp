// Mutation fuzzer for the host-side file formats of ancha_b200/csrc/hostio.cpp (manifest JSON,
// safetensors, WAV), built with AddressSanitizer / UBSan by test_host_formats_fuzz_cpu.py. A
// model package and an input track are untrusted files: every mutation must either parse or
// throw std::exception, with no sanitizer report.
// Usage: fuzz_host_formats ITERATIONS SEED SCRATCH_WAV_PATH manifest.json model.safetensors track.wav
#include "hostio.hpp"

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iterator>
#include <random>

using namespace ancha;

static std::string slurp(const char* p) {
    std::ifstream f(p, std::ios::binary);
    return std::string(std::istreambuf_iterator<char>(f), {});
}

static void mutate(std::string& b, std::mt19937_64& rng) {
    static const char* tokens[] = {"[", "{", "\"", "\\u12", "\\uzzzz", "1e999", "-1", "-41", "1e300",
                                   "9007199254740993", "18446744073709551615", "null", ",", ":", "}", "]"};
    const int muts = (int)(rng() % 6);
    for (int m = 0; m < muts && !b.empty(); ++m) {
        const size_t pos = rng() % b.size();
        switch (rng() % 7) {
            case 0: b[pos] ^= (char)(1u << (rng() % 8)); break;
            case 1: b[pos] = (char)rng(); break;
            case 2: b.resize(pos); break;
            case 3: b.insert(pos, 1, (char)rng()); break;
            case 4: b.erase(pos, 1); break;
            case 5: b.insert(pos, tokens[rng() % 16]); break;
            case 6: if (pos + 1 < b.size()) b.replace(pos, 1, std::string(1 + rng() % 400, b[pos])); break;
        }
    }
}

// Touch every node through the typed accessors.
static void walk(const Json& j) {
    switch (j.kind) {
        case Json::Number: try { (void)j.as_int(); } catch (const std::exception&) {} break;
        case Json::Array: for (const auto& v : j.arr) walk(v); break;
        case Json::Object: for (const auto& kv : j.obj) walk(kv.second); break;
        default: break;
    }
}

int main(int argc, char** argv) {
    if (argc != 7) return 2;
    const long iters = atol(argv[1]);
    std::mt19937_64 rng(strtoull(argv[2], nullptr, 10));
    const char* wav_path = argv[3];
    const std::string json = slurp(argv[4]), st = slurp(argv[5]), wav = slurp(argv[6]);
    long parsed[3] = {0, 0, 0}, thrown[3] = {0, 0, 0};
    // Directed cases: each must throw.
    auto throws = [](auto f) { try { f(); return false; } catch (const std::exception&) { return true; } };
    auto safetensors = [](const std::string& header, size_t data) {
        std::string b(8, '\0');
        for (int i = 0; i < 8; ++i) b[i] = (char)(header.size() >> (8 * i));
        return b + header + std::string(data, '\0');
    };
    const std::string wrap = safetensors(R"({"t":{"dtype":"F32","shape":[10],"data_offsets":[-41,-1]}})", 64);
    const std::string huge = safetensors(R"({"t":{"dtype":"F32","shape":[4611686018427387905],"data_offsets":[0,4]}})", 4);
    const std::string neg = safetensors(R"({"t":{"dtype":"F32","shape":[-1,-4],"data_offsets":[0,16]}})", 16);
    const bool directed[] = {
        throws([] { Json::parse(std::string(100000, '[')); }),          // nesting beyond the bound
        throws([] { (void)Json::parse("1e300").as_int(); }),            // no int64 value
        throws([] { (void)Json::parse("9007199254740994").as_int(); }), // past 2^53: not exact in a double
        throws([] { Json::parse(R"("\u12zz")"); }),                    // not four hex digits
        throws([&] { SafeTensors w(wrap); }),                            // offsets that wrap a size_t sum
        throws([&] { SafeTensors w(huge); (void)w.take("t", {4611686018427387905LL}); }),  // count · 4 wraps to 4
        throws([&] { SafeTensors w(neg); }),                             // negative dims
    };
    for (size_t k = 0; k < sizeof directed / sizeof directed[0]; ++k)
        if (!directed[k]) { fprintf(stderr, "directed case %zu was accepted\n", k); return 3; }
    for (long it = 0; it < iters; ++it) {
        std::string b = json;
        mutate(b, rng);
        try { const Json j = Json::parse(b); walk(j); (void)j.dump(); ++parsed[0]; }
        catch (const std::exception&) { ++thrown[0]; }

        b = st;
        mutate(b, rng);
        try {
            SafeTensors w(b);
            // Take every tensor the (mutated) header names, with the shape it states.
            uint64_t n = 0;
            for (int i = 0; i < 8; ++i) n |= (uint64_t)(uint8_t)b[i] << (8 * i);
            const Json h = Json::parse(b.substr(8, n));
            for (const auto& kv : h.obj) {
                if (kv.first == "__metadata__") continue;
                std::vector<int64_t> shape;
                for (const auto& d : kv.second.at("shape").arr) shape.push_back(d.as_int());
                try { (void)w.take(kv.first, shape); } catch (const std::exception&) {}
            }
            try { (void)w.finish(); } catch (const std::exception&) {}
            ++parsed[1];
        } catch (const std::exception&) { ++thrown[1]; }

        if (it % 4 == 0) {
            b = wav;
            mutate(b, rng);
            {
                std::ofstream f(wav_path, std::ios::binary | std::ios::trunc);
                f.write(b.data(), (std::streamsize)b.size());
            }
            try { const Audio a = read_wav(wav_path); (void)a.samples(); ++parsed[2]; }
            catch (const std::exception&) { ++thrown[2]; }
        }
    }
    printf("json %ld %ld safetensors %ld %ld wav %ld %ld\n", parsed[0], thrown[0], parsed[1], thrown[1], parsed[2],
           thrown[2]);
    return 0;
}
