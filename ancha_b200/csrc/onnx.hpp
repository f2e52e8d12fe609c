// ONNX model reading and the classic MDX executable graph (host side).
//
// parse_onnx decodes the protobuf wire format of the ModelProto subset the classic MDX
// executor of crates/ancha-models/src/mdx.rs reads (opset imports, graph nodes with INT /
// INTS / FLOAT attributes, FLOAT initializers as raw or float data, named inputs / outputs);
// MdxGraph::build restates Graph::from_bytes (mdx.rs:161-472): validation, BatchNormalization
// folding into its ConvTranspose producer and the instruction schedule with value lifetimes;
// MdxGraph::infer is the shape inference the executor runs before any launch.
#pragma once
#include <array>
#include <cstdint>
#include <string>
#include <vector>

namespace ancha {

using Shape4 = std::array<int64_t, 4>;

// Bounds on every value of a classic MDX graph (constants, the input, each op's output): with
// dimensions ≤ 2^30 and attributes ≤ 2^20, the per-axis indices the device kernels form
// (i·stride − pad + tap·dilation) fit in 32 bits; flat offsets are 64-bit.
constexpr int64_t kMdxMaxDim = int64_t(1) << 30;
constexpr int64_t kMdxMaxElements = int64_t(1) << 34;

// Element count of `n` dims when each lies in [1, kMdxMaxDim] and the count is at most
// kMdxMaxElements; −1 otherwise (no intermediate product can overflow).
int64_t mdx_checked_elements(const int64_t* dims, size_t n);

struct OnnxAttr {
    std::string name;
    int type = 0;
    int64_t i = 0;
    float f = 0.f;
    bool has_i = false, has_f = false;
    std::vector<int64_t> ints;
};

struct OnnxNode {
    std::vector<std::string> inputs, outputs;
    std::string name, op_type, domain;
    std::vector<OnnxAttr> attrs;
    const OnnxAttr* attr(const std::string& key) const;
};

struct OnnxTensor {
    std::string name;
    std::vector<int64_t> dims;
    int data_type = 0;
    bool external = false;
    std::vector<float> data;
};

struct OnnxModel {
    std::vector<std::pair<std::string, int64_t>> opset;  // (domain, version)
    bool has_graph = false;
    std::vector<OnnxNode> nodes;
    std::vector<OnnxTensor> initializers;
    int sparse_initializers = 0;
    std::vector<std::string> inputs, outputs;
};

OnnxModel parse_onnx(const uint8_t* data, size_t size);  // throws std::runtime_error

enum class MdxOp { Conv, ConvTranspose, Relu, Transpose, MatMul, Add, Mul, Bn };

struct MdxInstruction {
    MdxOp op = MdxOp::Relu;
    std::vector<int> inputs;  // value ids
    int output = -1;
    int stride[2] = {1, 1}, padding[2] = {0, 0}, dilation[2] = {1, 1}, padding_out[2] = {0, 0};
    int groups = 1;
    int perm[4] = {3, 2, 1, 0};
    float eps = 1e-5f;
    bool affine = false;             // the reference folds BatchNormalization to x·scale + shift
                                     // (optimized); the device always runs that form
    std::vector<float> scale, shift; // [channels] γ/√(var + ε), β − mean·scale
};

// Geometry of one Conv / ConvTranspose (NCHW; weights [co][ci/groups][kh][kw] for Conv and
// [ci][co/groups][kh][kw] for ConvTranspose), every field within kMdxMaxDim.
struct MdxConvShape {
    int n, ci, h, w, co, oh, ow, kh, kw, sh, sw, ph, pw, dh, dw, groups;
};

// Output geometry of a Conv / ConvTranspose instruction on input x and weight w (Burn's
// conv2d / conv_transpose2d size rules, in 64-bit arithmetic); false with `err` when the
// channels disagree, the output is empty or a size leaves the bounds above.
bool mdx_conv_shape(const MdxInstruction& ins, const Shape4& x, const Shape4& w, MdxConvShape& c, std::string& err);

struct MdxConstant {
    std::string name;
    int64_t shape[4] = {1, 1, 1, 1};  // initializer dims left-padded to four
    std::vector<float> data;
};

// Graph::from_bytes (mdx.rs:161-472). Value ids: the constants sorted by name, then the graph
// input, then one output per instruction in schedule order.
struct MdxGraph {
    std::vector<MdxConstant> constants;
    std::vector<MdxInstruction> instructions;
    std::vector<int> uses;  // consumers per value id, the graph output counted once more
    int input = -1, output = -1, values = 0;
    int folded_bn = 0, nodes = 0;
    static MdxGraph build(const OnnxModel& m, bool optimized);  // throws std::runtime_error
    // Shape of every value id for an NCHW input, op by op as Graph::forward applies them
    // (mdx.rs:474-568); false with `err` when an op's shapes disagree or a value leaves the
    // bounds above. Host-only.
    bool infer(const Shape4& in, std::vector<Shape4>& shapes, std::string& err) const;
};

}  // namespace ancha
