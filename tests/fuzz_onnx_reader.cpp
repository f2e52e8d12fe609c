// Mutation fuzzer for the classic MDX ONNX reader, graph builder and shape inference
// (ancha_b200/csrc/onnx.cpp), built with AddressSanitizer / UBSan by test_onnx_fuzz_cpu.py.
// Each iteration mutates a seed model (bit flips, byte changes, truncation, insertion,
// deletion, varint continuation bytes, huge length prefixes), builds it both ways and, when it
// builds, infers shapes for valid, extreme and invalid input shapes. Checked: no sanitizer
// report; every accepted value within the executor's bounds; every convolution's per-axis
// indices (i·stride − pad + tap·dilation) within 32 bits, as the device kernels form them.
// Usage: fuzz_onnx_reader ITERATIONS SEED model.onnx...
#include "onnx.hpp"
#include <climits>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iterator>
#include <random>
#include <stdexcept>
using namespace ancha;
static std::vector<uint8_t> slurp(const char* p) {
    std::ifstream f(p, std::ios::binary);
    return std::vector<uint8_t>(std::istreambuf_iterator<char>(f), {});
}
// The extreme per-axis index values of the conv / conv-transpose kernels, in 64-bit.
static void check_conv(const MdxConvShape& c, bool t) {
    auto fits = [](int64_t v) { return v >= INT32_MIN && v <= INT32_MAX; };
    bool ok = true;
    for (int64_t oy : {int64_t(0), int64_t(c.oh - 1)})
        for (int64_t ky : {int64_t(0), int64_t(c.kh - 1)})
            ok &= t ? fits(oy + c.ph - ky * c.dh) && fits(ky * c.dh) : fits(oy * c.sh - c.ph + ky * c.dh) && fits(oy * c.sh) && fits(ky * c.dh);
    for (int64_t ox : {int64_t(0), int64_t(c.ow - 1)})
        for (int64_t kx : {int64_t(0), int64_t(c.kw - 1)})
            ok &= t ? fits(ox + c.pw - kx * c.dw) && fits(kx * c.dw) : fits(ox * c.sw - c.pw + kx * c.dw) && fits(ox * c.sw) && fits(kx * c.dw);
    if (!ok) { fprintf(stderr, "32-bit index overflow in conv geometry\n"); abort(); }
}
int main(int argc, char** argv) {
    long iters = atol(argv[1]);
    std::mt19937_64 rng(atol(argv[2]));
    std::vector<std::vector<uint8_t>> seeds;
    for (int i = 3; i < argc; ++i) seeds.push_back(slurp(argv[i]));
    long ok = 0, rejected = 0, inferred = 0, convs = 0;
    const int64_t dims[] = {1, 2, 3, 4, 7, 8, 16, 64, 1000, 1 << 20, (int64_t)1 << 30, ((int64_t)1 << 30) + 1,
                            (int64_t)1 << 40, INT64_MAX, 0, -1};
    for (long it = 0; it < iters; ++it) {
        std::vector<uint8_t> b = seeds[rng() % seeds.size()];
        int muts = rng() % 9;
        for (int m = 0; m < muts && !b.empty(); ++m) {
            size_t pos = rng() % b.size();
            switch (rng() % 7) {
            case 0: b[pos] ^= (uint8_t)(1u << (rng() % 8)); break;
            case 1: b[pos] = (uint8_t)rng(); break;
            case 2: b.resize(pos); break;
            case 3: b.insert(b.begin() + pos, (uint8_t)rng()); break;
            case 4: b.erase(b.begin() + pos); break;
            case 5: b[pos] = (uint8_t)(0x80 | rng()); break;
            case 6: { static const uint8_t big[] = {0xff, 0xff, 0xff, 0xff, 0x0f};
                      b.insert(b.begin() + pos, big, big + 5); break; }
            }
        }
        if (b.empty()) continue;
        for (int opt = 0; opt < 2; ++opt) {
            MdxGraph g;
            try { g = MdxGraph::build(parse_onnx(b.data(), b.size()), opt != 0); ++ok; }
            catch (const std::exception&) { ++rejected; continue; }
            for (int k = 0; k < 6; ++k) {
                Shape4 in;
                for (int d = 0; d < 4; ++d) in[d] = (rng() % 3) ? dims[rng() % 9] : dims[rng() % 16];
                if (k == 0) in = {1, 4, 64, 32};
                std::vector<Shape4> shapes;
                std::string err;
                if (!g.infer(in, shapes, err)) continue;
                ++inferred;
                for (const auto& ins : g.instructions) {
                    if (ins.op != MdxOp::Conv && ins.op != MdxOp::ConvTranspose) continue;
                    MdxConvShape c;
                    if (!mdx_conv_shape(ins, shapes[ins.inputs[0]], shapes[ins.inputs[1]], c, err)) abort();
                    check_conv(c, ins.op == MdxOp::ConvTranspose);
                    ++convs;
                }
                for (const auto& sh : shapes)
                    if (mdx_checked_elements(sh.data(), 4) < 0) abort();
            }
        }
    }
    printf("iterations %ld accepted %ld rejected %ld inferred %ld convs %ld\n", iters, ok, rejected, inferred, convs);
    return 0;
}
