// Classic MDX graph executor, host side (mdx_exec.hpp): shape inference, constant upload and
// the schedule of Graph::forward (crates/ancha-models/src/mdx.rs:474-568).
#include <algorithm>
#include <stdexcept>
#include <string>

#include "mdx_exec.hpp"

namespace ancha {
namespace {

Shape4 strides_of(const Shape4& s) { return {s[1] * s[2] * s[3], s[2] * s[3], s[3], 1}; }

int64_t numel(const Shape4& s) { return s[0] * s[1] * s[2] * s[3]; }

std::string shape_text(const Shape4& s) {
    return "[" + std::to_string(s[0]) + ", " + std::to_string(s[1]) + ", " + std::to_string(s[2]) + ", " +
           std::to_string(s[3]) + "]";
}

// Conv / ConvTranspose geometry of instruction `ins` on input x and weight w; false when the
// shapes disagree (Burn's conv2d / conv_transpose2d rules).
bool conv_shape(const MdxInstruction& ins, const Shape4& x, const Shape4& w, MdxConvShape& c, std::string& err) {
    const bool t = ins.op == MdxOp::ConvTranspose;
    c.n = (int)x[0]; c.ci = (int)x[1]; c.h = (int)x[2]; c.w = (int)x[3];
    c.kh = (int)w[2]; c.kw = (int)w[3];
    c.sh = ins.stride[0]; c.sw = ins.stride[1]; c.ph = ins.padding[0]; c.pw = ins.padding[1];
    c.dh = ins.dilation[0]; c.dw = ins.dilation[1]; c.groups = ins.groups;
    if (t) {
        if (w[0] != x[1] || x[1] % ins.groups) { err = "conv_transpose channel mismatch"; return false; }
        c.co = (int)(w[1] * ins.groups);
        c.oh = (c.h - 1) * c.sh - 2 * c.ph + c.dh * (c.kh - 1) + ins.padding_out[0] + 1;
        c.ow = (c.w - 1) * c.sw - 2 * c.pw + c.dw * (c.kw - 1) + ins.padding_out[1] + 1;
    } else {
        if (w[1] * ins.groups != x[1] || w[0] % ins.groups) { err = "conv2d channel mismatch"; return false; }
        c.co = (int)w[0];
        c.oh = (c.h + 2 * c.ph - c.dh * (c.kh - 1) - 1) / c.sh + 1;
        c.ow = (c.w + 2 * c.pw - c.dw * (c.kw - 1) - 1) / c.sw + 1;
    }
    if (c.oh <= 0 || c.ow <= 0) { err = "convolution output is empty"; return false; }
    return true;
}

bool broadcast(const Shape4& a, const Shape4& b, Shape4& out) {
    for (int d = 0; d < 4; ++d) {
        if (a[d] != b[d] && a[d] != 1 && b[d] != 1) return false;
        out[d] = std::max(a[d], b[d]);
    }
    return true;
}

template <typename T>
void upload(DevBuf& d, const std::vector<T>& v) {
    d.alloc(std::max<size_t>(v.size(), 1) * sizeof(T));
    if (!v.empty() && cudaMemcpy(d.p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess)
        throw std::runtime_error("cudaMemcpy of an MDX constant");
}

}  // namespace

std::unique_ptr<MdxModel> MdxModel::load(const uint8_t* onnx, size_t bytes, bool optimized, int device) {
    std::unique_ptr<MdxModel> m(new MdxModel());
    m->graph = MdxGraph::build(parse_onnx(onnx, bytes), optimized);  // before any device work
    if (cudaSetDevice(device) != cudaSuccess) throw std::runtime_error("cudaSetDevice");
    m->device = device;
    m->constants_.resize(m->graph.constants.size());
    for (size_t i = 0; i < m->graph.constants.size(); ++i) upload(m->constants_[i], m->graph.constants[i].data);
    m->bn_scale_.resize(m->graph.instructions.size());
    m->bn_shift_.resize(m->graph.instructions.size());
    for (size_t i = 0; i < m->graph.instructions.size(); ++i) {
        const MdxInstruction& ins = m->graph.instructions[i];
        if (ins.op != MdxOp::Bn) continue;
        upload(m->bn_scale_[i], ins.scale);
        upload(m->bn_shift_[i], ins.shift);
    }
    return m;
}

int MdxModel::infer(const Shape4& in, std::vector<Shape4>& shapes) const {
    if (std::any_of(in.begin(), in.end(), [](int64_t v) { return v <= 0; }))
        return fail(ANCHA_E_INVALID, "MDX graph input shape must be positive");
    shapes.assign(graph.values, Shape4{0, 0, 0, 0});
    for (size_t i = 0; i < graph.constants.size(); ++i)
        for (int d = 0; d < 4; ++d) shapes[i][d] = graph.constants[i].shape[d];
    shapes[graph.input] = in;
    for (const MdxInstruction& ins : graph.instructions) {
        const Shape4& a = shapes[ins.inputs[0]];
        Shape4 out = a;
        std::string err;
        switch (ins.op) {
            case MdxOp::Conv:
            case MdxOp::ConvTranspose: {
                MdxConvShape c;
                if (!conv_shape(ins, a, shapes[ins.inputs[1]], c, err)) return fail(ANCHA_E_INVALID, err);
                if (ins.inputs.size() == 3 && numel(shapes[ins.inputs[2]]) != c.co)
                    return fail(ANCHA_E_INVALID, "convolution bias length mismatch");
                out = {c.n, c.co, c.oh, c.ow};
                break;
            }
            case MdxOp::Relu: break;
            case MdxOp::Transpose:
                for (int d = 0; d < 4; ++d) out[d] = a[ins.perm[d]];
                break;
            case MdxOp::MatMul: {
                const Shape4& b = shapes[ins.inputs[1]];
                if (a[3] != b[2]) return fail(ANCHA_E_INVALID, "MatMul inner dimensions " + shape_text(a) + " · " + shape_text(b));
                for (int d = 0; d < 2; ++d) {
                    if (a[d] != b[d] && a[d] != 1 && b[d] != 1)
                        return fail(ANCHA_E_INVALID, "MatMul batch dimensions do not broadcast");
                    out[d] = std::max(a[d], b[d]);
                }
                out[2] = a[2];
                out[3] = b[3];
                break;
            }
            case MdxOp::Add:
            case MdxOp::Mul:
                if (!broadcast(a, shapes[ins.inputs[1]], out))
                    return fail(ANCHA_E_INVALID, "shapes " + shape_text(a) + " and " +
                                                     shape_text(shapes[ins.inputs[1]]) + " do not broadcast");
                break;
            case MdxOp::Bn:
                if (a[1] != (int64_t)ins.scale.size()) return fail(ANCHA_E_INVALID, "BatchNormalization channel mismatch");
                break;
        }
        if (numel(out) <= 0 || numel(out) > (int64_t)1 << 34) return fail(ANCHA_E_INVALID, "MDX value size out of range");
        shapes[ins.output] = out;
    }
    return ANCHA_OK;
}

int MdxModel::output_shape(const Shape4& in, Shape4& out) const {
    std::vector<Shape4> shapes;
    ANCHA_TRY(infer(in, shapes));
    out = shapes[graph.output];
    return ANCHA_OK;
}

int MdxModel::forward(const float* x, const Shape4& in, float* out, const volatile int* cancel, cudaStream_t s) {
    std::vector<Shape4> shapes;
    ANCHA_TRY(infer(in, shapes));
    ANCHA_CUDA(cudaSetDevice(device));
    const int nconst = (int)graph.constants.size();
    std::vector<float*> values(graph.values, nullptr);
    for (int i = 0; i < nconst; ++i) values[i] = constants_[i].as<float>();
    values[graph.input] = const_cast<float*>(x);
    std::vector<int> uses = graph.uses;
    auto owned = [&](int v) { return v > graph.input; };  // instruction outputs
    auto release_all = [&] {
        for (int v = graph.input + 1; v < graph.values; ++v)
            if (values[v]) {
                cudaFreeAsync(values[v], s);
                values[v] = nullptr;
            }
    };
    int st = ANCHA_OK;
    for (size_t k = 0; k < graph.instructions.size() && st == ANCHA_OK; ++k) {
        if (cancel && *cancel) { st = fail(ANCHA_E_CANCELLED, "task cancelled"); break; }
        const MdxInstruction& ins = graph.instructions[k];
        const Shape4& os = shapes[ins.output];
        float* y = nullptr;
        if (cudaMallocAsync(reinterpret_cast<void**>(&y), (size_t)numel(os) * sizeof(float), s) != cudaSuccess) {
            st = fail(ANCHA_E_CUDA, "cudaMallocAsync of an MDX value");
            break;
        }
        values[ins.output] = y;
        const Shape4& a = shapes[ins.inputs[0]];
        const float* va = values[ins.inputs[0]];
        switch (ins.op) {
            case MdxOp::Conv:
            case MdxOp::ConvTranspose: {
                MdxConvShape c;
                std::string err;
                conv_shape(ins, a, shapes[ins.inputs[1]], c, err);
                st = mdx_conv2d(va, values[ins.inputs[1]], ins.inputs.size() == 3 ? values[ins.inputs[2]] : nullptr, y,
                                c, ins.op == MdxOp::ConvTranspose, s);
                break;
            }
            case MdxOp::Relu:
            case MdxOp::Add:
            case MdxOp::Mul:
            case MdxOp::Bn: {
                MdxEwise e{};
                e.op = ins.op == MdxOp::Relu ? 0 : ins.op == MdxOp::Add ? 1 : ins.op == MdxOp::Mul ? 2 : 3;
                const Shape4 sa = strides_of(a);
                for (int d = 0; d < 4; ++d) {
                    e.out[d] = os[d];
                    e.sa[d] = a[d] == 1 ? 0 : sa[d];
                }
                const float* vb = nullptr;
                if (e.op == 1 || e.op == 2) {
                    const Shape4& b = shapes[ins.inputs[1]];
                    const Shape4 sb = strides_of(b);
                    for (int d = 0; d < 4; ++d) e.sb[d] = b[d] == 1 ? 0 : sb[d];
                    vb = values[ins.inputs[1]];
                } else if (e.op == 3) {
                    e.sb[1] = 1;  // channel index into scale / shift
                    e.scale = bn_scale_[k].as<float>();
                    e.shift = bn_shift_[k].as<float>();
                }
                st = mdx_ewise(va, vb, y, e, s);
                break;
            }
            case MdxOp::Transpose: {
                MdxPermute p{};
                const Shape4 sa = strides_of(a);
                for (int d = 0; d < 4; ++d) {
                    p.out[d] = os[d];
                    p.stride[d] = sa[ins.perm[d]];
                }
                st = mdx_permute(va, y, p, s);
                break;
            }
            case MdxOp::MatMul: {
                const Shape4& b = shapes[ins.inputs[1]];
                MdxMatmul mm{};
                mm.batch[0] = os[0];
                mm.batch[1] = os[1];
                mm.sa[0] = a[0] == 1 ? 0 : a[1] * a[2] * a[3];
                mm.sa[1] = a[1] == 1 ? 0 : a[2] * a[3];
                mm.sb[0] = b[0] == 1 ? 0 : b[1] * b[2] * b[3];
                mm.sb[1] = b[1] == 1 ? 0 : b[2] * b[3];
                mm.m = (int)a[2];
                mm.k = (int)a[3];
                mm.n = (int)b[3];
                st = mdx_matmul(va, values[ins.inputs[1]], y, mm, s);
                break;
            }
        }
        // Release inputs whose last consumer this was (mdx.rs:556-561).
        for (int v : ins.inputs)
            if (--uses[v] == 0 && owned(v) && values[v]) {
                cudaFreeAsync(values[v], s);
                values[v] = nullptr;
            }
    }
    if (st == ANCHA_OK) {
        const Shape4& os = shapes[graph.output];
        const float* src = values[graph.output];
        if (cudaMemcpyAsync(out, src, (size_t)numel(os) * sizeof(float), cudaMemcpyDeviceToDevice, s) != cudaSuccess)
            st = fail(ANCHA_E_CUDA, "copy of the MDX graph output");
    }
    release_all();
    return st;
}

}  // namespace ancha
