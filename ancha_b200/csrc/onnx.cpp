// ONNX reading and the classic MDX graph builder (onnx.hpp).
#include "onnx.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <set>
#include <stdexcept>

namespace ancha {
namespace {

[[noreturn]] void bad(const std::string& m) { throw std::runtime_error(m); }

// One protobuf message: fields are visited in order; length-delimited payloads are views into
// the caller's buffer.
struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    Reader(const uint8_t* b, size_t n) : p(b), end(b + n) {}
    bool done() const { return p >= end; }
    uint64_t varint() {
        uint64_t v = 0;
        for (int shift = 0; shift < 64; shift += 7) {
            if (p >= end) bad("truncated protobuf varint");
            const uint8_t b = *p++;
            v |= (uint64_t)(b & 0x7F) << shift;
            if (!(b & 0x80)) return v;
        }
        bad("invalid protobuf varint");
    }
    struct Field {
        uint32_t number, wire;
        uint64_t v;                 // varint / fixed values
        const uint8_t* data = nullptr;  // length-delimited payload
        size_t size = 0;
    };
    Field next() {
        Field f{};
        const uint64_t key = varint();
        f.number = (uint32_t)(key >> 3);
        f.wire = (uint32_t)(key & 7);
        switch (f.wire) {
            case 0: f.v = varint(); break;
            case 1:
                if (end - p < 8) bad("truncated protobuf fixed64");
                std::memcpy(&f.v, p, 8);
                p += 8;
                break;
            case 2: {
                const uint64_t n = varint();
                if ((uint64_t)(end - p) < n) bad("truncated protobuf field");
                f.data = p;
                f.size = (size_t)n;
                p += n;
                break;
            }
            case 5: {
                if (end - p < 4) bad("truncated protobuf fixed32");
                uint32_t v32;
                std::memcpy(&v32, p, 4);
                f.v = v32;
                p += 4;
                break;
            }
            default: bad("unsupported protobuf wire type");
        }
        return f;
    }
};

std::string text(const Reader::Field& f) {
    if (f.wire != 2) bad("expected a string field");
    return std::string(reinterpret_cast<const char*>(f.data), f.size);
}

void append_ints(const Reader::Field& f, std::vector<int64_t>& out) {
    if (f.wire == 2) {
        Reader r(f.data, f.size);
        while (!r.done()) out.push_back((int64_t)r.varint());
    } else if (f.wire == 0) {
        out.push_back((int64_t)f.v);
    } else {
        bad("expected an integer field");
    }
}

float as_float(uint64_t bits) {
    const uint32_t b = (uint32_t)bits;
    float f;
    std::memcpy(&f, &b, 4);
    return f;
}

OnnxAttr parse_attr(const uint8_t* d, size_t n) {
    OnnxAttr a;
    Reader r(d, n);
    while (!r.done()) {
        const auto f = r.next();
        switch (f.number) {
            case 1: a.name = text(f); break;
            case 20: a.type = (int)f.v; break;
            case 3: a.i = (int64_t)f.v; a.has_i = true; break;
            case 2:
                if (f.wire != 5) bad("invalid float attribute");
                a.f = as_float(f.v);
                a.has_f = true;
                break;
            case 8: append_ints(f, a.ints); break;
            default: break;
        }
    }
    return a;
}

OnnxNode parse_node(const uint8_t* d, size_t n) {
    OnnxNode node;
    Reader r(d, n);
    while (!r.done()) {
        const auto f = r.next();
        switch (f.number) {
            case 1: node.inputs.push_back(text(f)); break;
            case 2: node.outputs.push_back(text(f)); break;
            case 3: node.name = text(f); break;
            case 4: node.op_type = text(f); break;
            case 7: node.domain = text(f); break;
            case 5: node.attrs.push_back(parse_attr(f.data, f.size)); break;
            default: break;
        }
    }
    return node;
}

OnnxTensor parse_tensor(const uint8_t* d, size_t n) {
    OnnxTensor t;
    Reader r(d, n);
    const uint8_t* raw = nullptr;
    size_t raw_size = 0;
    std::vector<float> floats;
    while (!r.done()) {
        const auto f = r.next();
        switch (f.number) {
            case 1: append_ints(f, t.dims); break;
            case 2: t.data_type = (int)f.v; break;
            case 8: t.name = text(f); break;
            case 9: raw = f.data; raw_size = f.size; break;
            case 4:
                if (f.wire == 2) {
                    if (f.size % 4) bad("invalid packed float data");
                    for (size_t i = 0; i < f.size; i += 4) {
                        uint32_t b;
                        std::memcpy(&b, f.data + i, 4);
                        floats.push_back(as_float(b));
                    }
                } else if (f.wire == 5) {
                    floats.push_back(as_float(f.v));
                }
                break;
            case 14: t.external = f.v == 1; break;
            default: break;
        }
    }
    if (raw) {
        if (raw_size % 4) bad("invalid raw tensor data");
        t.data.resize(raw_size / 4);
        if (raw_size) std::memcpy(t.data.data(), raw, raw_size);  // little-endian host, as ONNX stores it
    } else {
        t.data = std::move(floats);
    }
    return t;
}

std::string value_name(const uint8_t* d, size_t n) {
    Reader r(d, n);
    while (!r.done()) {
        const auto f = r.next();
        if (f.number == 1) return text(f);
    }
    return "";
}

int64_t int_attr(const OnnxNode& n, const char* key, int64_t def) {
    const OnnxAttr* a = n.attr(key);
    return a && a->has_i ? a->i : def;
}

std::vector<int64_t> ints_attr(const OnnxNode& n, const char* key, std::vector<int64_t> def) {
    const OnnxAttr* a = n.attr(key);
    return a ? a->ints : def;
}

float float_attr(const OnnxNode& n, const char* key, float def) {
    const OnnxAttr* a = n.attr(key);
    return a && a->has_f ? a->f : def;
}

void pair(const std::vector<int64_t>& v, bool positive, int out[2]) {
    if (v.size() != 2) bad("invalid pair attribute");
    for (int i = 0; i < 2; ++i) {
        if (v[i] < (positive ? 1 : 0) || v[i] > (1 << 20)) bad("invalid pair attribute");
        out[i] = (int)v[i];
    }
}

std::string shape_text(const Shape4& s) {
    return "[" + std::to_string(s[0]) + ", " + std::to_string(s[1]) + ", " + std::to_string(s[2]) + ", " +
           std::to_string(s[3]) + "]";
}

}  // namespace

int64_t mdx_checked_elements(const int64_t* dims, size_t n) {
    int64_t count = 1;
    for (size_t i = 0; i < n; ++i) {
        if (dims[i] < 1 || dims[i] > kMdxMaxDim || count > kMdxMaxElements / dims[i]) return -1;
        count *= dims[i];
    }
    return count;
}

bool mdx_conv_shape(const MdxInstruction& ins, const Shape4& x, const Shape4& w, MdxConvShape& c, std::string& err) {
    // Inputs are values within kMdxMaxDim and attributes within 2^20, so no product below
    // exceeds 2^51.
    const int64_t g = ins.groups, kh = w[2], kw = w[3];
    int64_t co, oh, ow;
    if (ins.op == MdxOp::ConvTranspose) {
        if (w[0] != x[1] || x[1] % g) { err = "conv_transpose channel mismatch"; return false; }
        co = w[1] * g;
        oh = (x[2] - 1) * ins.stride[0] - 2 * (int64_t)ins.padding[0] + ins.dilation[0] * (kh - 1) + ins.padding_out[0] + 1;
        ow = (x[3] - 1) * ins.stride[1] - 2 * (int64_t)ins.padding[1] + ins.dilation[1] * (kw - 1) + ins.padding_out[1] + 1;
    } else {
        if (w[1] * g != x[1] || w[0] % g) { err = "conv2d channel mismatch"; return false; }
        co = w[0];
        // Positions the kernel's first tap can take; negative when the dilated kernel is wider
        // than the padded input (an empty output, not one truncated towards zero).
        const int64_t span_h = x[2] + 2 * (int64_t)ins.padding[0] - ins.dilation[0] * (kh - 1) - 1;
        const int64_t span_w = x[3] + 2 * (int64_t)ins.padding[1] - ins.dilation[1] * (kw - 1) - 1;
        oh = span_h < 0 ? 0 : span_h / ins.stride[0] + 1;
        ow = span_w < 0 ? 0 : span_w / ins.stride[1] + 1;
    }
    if (oh <= 0 || ow <= 0) { err = "convolution output is empty"; return false; }
    if (co > kMdxMaxDim || oh > kMdxMaxDim || ow > kMdxMaxDim) { err = "convolution output too large"; return false; }
    c.n = (int)x[0]; c.ci = (int)x[1]; c.h = (int)x[2]; c.w = (int)x[3];
    c.co = (int)co; c.oh = (int)oh; c.ow = (int)ow; c.kh = (int)kh; c.kw = (int)kw;
    c.sh = ins.stride[0]; c.sw = ins.stride[1]; c.ph = ins.padding[0]; c.pw = ins.padding[1];
    c.dh = ins.dilation[0]; c.dw = ins.dilation[1]; c.groups = ins.groups;
    return true;
}

bool MdxGraph::infer(const Shape4& in, std::vector<Shape4>& shapes, std::string& err) const {
    if (std::any_of(in.begin(), in.end(), [](int64_t v) { return v <= 0; })) {
        err = "MDX graph input shape must be positive";
        return false;
    }
    if (mdx_checked_elements(in.data(), 4) < 0) {
        err = "MDX graph input shape " + shape_text(in) + " too large";
        return false;
    }
    shapes.assign(values, Shape4{0, 0, 0, 0});
    for (size_t i = 0; i < constants.size(); ++i)
        for (int d = 0; d < 4; ++d) shapes[i][d] = constants[i].shape[d];
    shapes[input] = in;
    for (const MdxInstruction& ins : instructions) {
        const Shape4& a = shapes[ins.inputs[0]];
        Shape4 out = a;
        switch (ins.op) {
            case MdxOp::Conv:
            case MdxOp::ConvTranspose: {
                MdxConvShape c;
                if (!mdx_conv_shape(ins, a, shapes[ins.inputs[1]], c, err)) return false;
                if (ins.inputs.size() == 3 && mdx_checked_elements(shapes[ins.inputs[2]].data(), 4) != c.co) {
                    err = "convolution bias length mismatch";
                    return false;
                }
                out = {c.n, c.co, c.oh, c.ow};
                break;
            }
            case MdxOp::Relu: break;
            case MdxOp::Transpose:
                for (int d = 0; d < 4; ++d) out[d] = a[ins.perm[d]];
                break;
            case MdxOp::MatMul: {
                const Shape4& b = shapes[ins.inputs[1]];
                if (a[3] != b[2]) {
                    err = "MatMul inner dimensions " + shape_text(a) + " · " + shape_text(b);
                    return false;
                }
                for (int d = 0; d < 2; ++d) {
                    if (a[d] != b[d] && a[d] != 1 && b[d] != 1) {
                        err = "MatMul batch dimensions do not broadcast";
                        return false;
                    }
                    out[d] = std::max(a[d], b[d]);
                }
                out[2] = a[2];
                out[3] = b[3];
                break;
            }
            case MdxOp::Add:
            case MdxOp::Mul: {
                const Shape4& b = shapes[ins.inputs[1]];
                for (int d = 0; d < 4; ++d) {
                    if (a[d] != b[d] && a[d] != 1 && b[d] != 1) {
                        err = "shapes " + shape_text(a) + " and " + shape_text(b) + " do not broadcast";
                        return false;
                    }
                    out[d] = std::max(a[d], b[d]);
                }
                break;
            }
            case MdxOp::Bn:
                if (a[1] != (int64_t)ins.scale.size()) {
                    err = "BatchNormalization channel mismatch";
                    return false;
                }
                break;
        }
        if (mdx_checked_elements(out.data(), 4) < 0) {
            err = "MDX value size out of range";
            return false;
        }
        shapes[ins.output] = out;
    }
    return true;
}

const OnnxAttr* OnnxNode::attr(const std::string& key) const {
    for (const auto& a : attrs)
        if (a.name == key) return &a;
    return nullptr;
}

OnnxModel parse_onnx(const uint8_t* data, size_t size) {
    OnnxModel m;
    Reader r(data, size);
    while (!r.done()) {
        const auto f = r.next();
        if (f.number == 8 && f.wire == 2) {
            std::string domain;
            int64_t version = 0;
            Reader o(f.data, f.size);
            while (!o.done()) {
                const auto g = o.next();
                if (g.number == 1) domain = text(g);
                if (g.number == 2) version = (int64_t)g.v;
            }
            m.opset.emplace_back(domain, version);
        } else if (f.number == 7 && f.wire == 2) {
            m.has_graph = true;
            Reader g(f.data, f.size);
            while (!g.done()) {
                const auto h = g.next();
                if (h.wire != 2) continue;
                switch (h.number) {
                    case 1: m.nodes.push_back(parse_node(h.data, h.size)); break;
                    case 5: m.initializers.push_back(parse_tensor(h.data, h.size)); break;
                    case 15: ++m.sparse_initializers; break;
                    case 11: m.inputs.push_back(value_name(h.data, h.size)); break;
                    case 12: m.outputs.push_back(value_name(h.data, h.size)); break;
                    default: break;
                }
            }
        }
    }
    return m;
}

MdxGraph MdxGraph::build(const OnnxModel& m, bool optimized) {
    if (m.opset.size() != 1 || !m.opset[0].first.empty() || m.opset[0].second != 13)
        bad("classic MDX executor requires ONNX opset 13");
    if (!m.has_graph) bad("missing ONNX graph");
    if (m.inputs.size() != 1 || m.outputs.size() != 1 || m.sparse_initializers)
        bad("expected one input and one output, no sparse initializers");
    // Initializers: FLOAT, at most four positive dims (left-padded to four), finite.
    std::map<std::string, MdxConstant> raw;
    for (const OnnxTensor& t : m.initializers) {
        if (t.data_type != 1 || t.dims.size() > 4 || t.external ||
            std::any_of(t.dims.begin(), t.dims.end(), [](int64_t v) { return v <= 0; }))
            bad("unsupported initializer " + t.name);
        MdxConstant c;
        c.name = t.name;
        for (size_t i = 0; i < t.dims.size(); ++i) c.shape[4 - t.dims.size() + i] = t.dims[i];
        const int64_t count = mdx_checked_elements(c.shape, 4);  // −1 when out of bounds
        if (count < 0 || (int64_t)t.data.size() != count ||
            std::any_of(t.data.begin(), t.data.end(), [](float v) { return !std::isfinite(v); }))
            bad("invalid initializer " + t.name);
        c.data = t.data;
        if (!raw.emplace(t.name, std::move(c)).second) bad("duplicate initializer");
    }
    std::map<std::string, int> consumers;
    for (const auto& n : m.nodes)
        for (const auto& s : n.inputs) ++consumers[s];
    auto stats = [&](const OnnxNode& bn, std::vector<float>& scale, std::vector<float>& shift, float eps) {
        const auto& gamma = raw.at(bn.inputs[1]).data;
        const auto& beta = raw.at(bn.inputs[2]).data;
        const auto& mean = raw.at(bn.inputs[3]).data;
        const auto& var = raw.at(bn.inputs[4]).data;
        if (gamma.size() != beta.size() || gamma.size() != mean.size() || gamma.size() != var.size() ||
            std::any_of(var.begin(), var.end(), [](float v) { return v < 0.f; }))
            bad("invalid BN statistics");
        scale.resize(gamma.size());
        shift.resize(gamma.size());
        for (size_t c = 0; c < gamma.size(); ++c) {
            scale[c] = gamma[c] / std::sqrt(var[c] + eps);
            shift[c] = beta[c] - mean[c] * scale[c];
        }
    };
    std::set<size_t> skipped;
    std::map<size_t, std::string> redirected;
    MdxGraph g;
    if (optimized) {
        // A BatchNormalization whose only producer is a ConvTranspose folds into its weights
        // and bias (mdx.rs:216-294).
        for (size_t i = 0; i < m.nodes.size(); ++i) {
            const OnnxNode& n = m.nodes[i];
            if (n.op_type != "ConvTranspose" || n.outputs.size() != 1 || consumers[n.outputs[0]] != 1 ||
                m.outputs[0] == n.outputs[0])
                continue;
            size_t j = 0;
            for (; j < m.nodes.size(); ++j)
                if (m.nodes[j].op_type == "BatchNormalization" && !m.nodes[j].inputs.empty() &&
                    m.nodes[j].inputs[0] == n.outputs[0])
                    break;
            if (j == m.nodes.size()) continue;
            const OnnxNode& bn = m.nodes[j];
            if (bn.inputs.size() != 5 || bn.outputs.size() != 1 || int_attr(bn, "training_mode", 0) != 0)
                bad("unsupported BN");
            if (n.inputs.size() != 3 || int_attr(n, "group", 1) != 1)
                bad("folding expects ungrouped transposed convolution with bias");
            for (int k = 1; k < 5; ++k)
                if (!raw.count(bn.inputs[k])) bad("BN statistics must be initializers");
            if (!raw.count(n.inputs[1]) || !raw.count(n.inputs[2])) bad("folding expects constant weights");
            const float eps = float_attr(bn, "epsilon", 1e-5f);
            if (!(eps > 0.f) || !std::isfinite(eps)) bad("invalid BN epsilon");
            std::vector<float> scale, shift;
            stats(bn, scale, shift, eps);
            const MdxConstant& w = raw.at(n.inputs[1]);
            const int64_t ci = w.shape[0], co = w.shape[1], kk = w.shape[2] * w.shape[3];
            if (co != (int64_t)scale.size()) bad("BN / ConvTranspose channel mismatch");
            MdxConstant fw = w;
            fw.name = "__ancha_fold_" + std::to_string(i) + "_weight";
            for (int64_t a = 0; a < ci; ++a)
                for (int64_t o = 0; o < co; ++o)
                    for (int64_t k = 0; k < kk; ++k) fw.data[(a * co + o) * kk + k] *= scale[o];
            const MdxConstant& b = raw.at(n.inputs[2]);
            if ((int64_t)b.data.size() != co) bad("invalid transpose bias");
            MdxConstant fb;
            fb.name = "__ancha_fold_" + std::to_string(i) + "_bias";
            fb.shape[3] = co;
            fb.data.resize(co);
            for (int64_t o = 0; o < co; ++o) fb.data[o] = b.data[o] * scale[o] + shift[o];
            raw[fw.name] = std::move(fw);
            raw[fb.name] = std::move(fb);
            skipped.insert(j);
            redirected[i] = bn.outputs[0];
            ++g.folded_bn;
        }
    }
    // Value ids: constants in name order, the input, then each instruction's output.
    std::map<std::string, int> ids;
    for (auto& kv : raw) {
        ids[kv.first] = (int)g.constants.size();
        g.constants.push_back(kv.second);
    }
    g.input = (int)g.constants.size();
    ids[m.inputs[0]] = g.input;
    int next = g.input + 1;
    for (size_t i = 0; i < m.nodes.size(); ++i) {
        if (skipped.count(i)) continue;
        const OnnxNode& n = m.nodes[i];
        if (!n.domain.empty() || n.outputs.size() != 1) bad("unsupported node domain or multi-output");
        static const std::set<std::string> conv_attrs = {"dilations", "group", "kernel_shape", "pads", "strides",
                                                         "output_padding"};
        static const std::set<std::string> bn_attrs = {"epsilon", "momentum", "training_mode"};
        static const std::set<std::string> transpose_attrs = {"perm"};
        static const std::set<std::string> none;
        const bool conv = n.op_type == "Conv" || n.op_type == "ConvTranspose";
        const std::set<std::string>& allowed = conv ? conv_attrs
                                               : n.op_type == "BatchNormalization" ? bn_attrs
                                               : n.op_type == "Transpose" ? transpose_attrs : none;
        for (const auto& a : n.attrs)
            if (!allowed.count(a.name)) bad("unsupported attribute in " + n.name);
        MdxInstruction ins;
        for (const auto& s : n.inputs) {
            auto it = ids.find(s);
            if (it == ids.end()) bad("unknown input " + s);
            ins.inputs.push_back(it->second);
        }
        if (conv) {
            if (ins.inputs.size() != 2 && ins.inputs.size() != 3) bad("invalid conv inputs");
            const auto pads = ints_attr(n, "pads", {0, 0, 0, 0});
            if (pads.size() != 4 || pads[0] != pads[2] || pads[1] != pads[3])
                bad("asymmetric convolution unsupported");
            const int64_t groups = int_attr(n, "group", 1);
            if (groups <= 0 || groups > (1 << 20)) bad("invalid groups");
            ins.op = n.op_type == "Conv" ? MdxOp::Conv : MdxOp::ConvTranspose;
            if (redirected.count(i)) {
                ins.inputs[1] = ids.at("__ancha_fold_" + std::to_string(i) + "_weight");
                ins.inputs[2] = ids.at("__ancha_fold_" + std::to_string(i) + "_bias");
            }
            pair(ints_attr(n, "strides", {1, 1}), true, ins.stride);
            pair({pads[0], pads[1]}, false, ins.padding);
            pair(ints_attr(n, "dilations", {1, 1}), true, ins.dilation);
            pair(ints_attr(n, "output_padding", {0, 0}), false, ins.padding_out);
            ins.groups = (int)groups;
        } else if (n.op_type == "Relu") {
            if (ins.inputs.size() != 1) bad("invalid Relu inputs");
            ins.op = MdxOp::Relu;
        } else if (n.op_type == "Transpose") {
            if (ins.inputs.size() != 1) bad("invalid transpose inputs");
            const auto p = ints_attr(n, "perm", {3, 2, 1, 0});
            std::set<int64_t> s(p.begin(), p.end());
            if (p.size() != 4 || s != std::set<int64_t>{0, 1, 2, 3}) bad("invalid permutation");
            for (int k = 0; k < 4; ++k) ins.perm[k] = (int)p[k];
            ins.op = MdxOp::Transpose;
        } else if (n.op_type == "MatMul" || n.op_type == "Add" || n.op_type == "Mul") {
            if (ins.inputs.size() != 2) bad("invalid binary inputs");
            ins.op = n.op_type == "MatMul" ? MdxOp::MatMul : n.op_type == "Add" ? MdxOp::Add : MdxOp::Mul;
        } else if (n.op_type == "BatchNormalization") {
            if (ins.inputs.size() != 5 || int_attr(n, "training_mode", 0) != 0) bad("only eval BN supported");
            for (int k = 1; k < 5; ++k)
                if (!raw.count(n.inputs[k])) bad("BN statistics must be initializers");
            ins.eps = float_attr(n, "epsilon", 1e-5f);
            if (!std::isfinite(ins.eps) || !(ins.eps > 0.f)) bad("invalid BN epsilon");
            ins.op = MdxOp::Bn;
            stats(n, ins.scale, ins.shift, ins.eps);
            ins.affine = optimized;
        } else {
            bad("unsupported ONNX operation " + n.op_type + " at " + n.name);
        }
        const std::string name = redirected.count(i) ? redirected[i] : n.outputs[0];
        if (!ids.emplace(name, next).second) bad("duplicate ONNX value");
        ins.output = next++;
        g.instructions.push_back(std::move(ins));
    }
    auto out = ids.find(m.outputs[0]);
    if (out == ids.end()) bad("graph output missing");
    g.output = out->second;
    g.values = next;
    g.uses.assign(next, 0);
    for (const auto& ins : g.instructions)
        for (int v : ins.inputs) ++g.uses[v];
    ++g.uses[g.output];
    g.nodes = (int)m.nodes.size();
    return g;
}

}  // namespace ancha
