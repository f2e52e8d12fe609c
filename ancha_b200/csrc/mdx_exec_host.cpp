// Classic MDX graph executor, host side (mdx_exec.hpp): constant upload and the schedule of
// Graph::forward (crates/ancha-models/src/mdx.rs:474-568) over the shapes of MdxGraph::infer.
#include <algorithm>
#include <chrono>
#include <climits>
#include <cmath>
#include <stdexcept>
#include <string>

#include "mdx_exec.hpp"
#include "rowops.cuh"

namespace ancha {
namespace {

Shape4 strides_of(const Shape4& s) { return {s[1] * s[2] * s[3], s[2] * s[3], s[3], 1}; }

int64_t numel(const Shape4& s) { return s[0] * s[1] * s[2] * s[3]; }

template <typename T>
void upload(DevBuf& d, const std::vector<T>& v) {
    d.alloc(std::max<size_t>(v.size(), 1) * sizeof(T));
    if (!v.empty() && cudaMemcpy(d.p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess)
        throw std::runtime_error("cudaMemcpy of an MDX constant");
}

void upload_elt(DevBuf& d, const std::vector<float>& v, int elt) {
    if (elt == ELT_F32) return upload(d, v);
    if (elt == ELT_BF16) {
        std::vector<__nv_bfloat16> h(v.size());
        for (size_t i = 0; i < v.size(); ++i) h[i] = __float2bfloat16_rn(v[i]);
        return upload(d, h);
    }
    std::vector<__half> h(v.size());
    for (size_t i = 0; i < v.size(); ++i) h[i] = __float2half_rn(v[i]);
    upload(d, h);
}

// The patch-gather geometries (mdx_pack): 1×1 stride 1, 3×3 stride 1 padding 1, 2×2 stride 2,
// of an ungrouped, undilated Conv whose kernel is kh × kw.
bool gemm_geometry(const MdxInstruction& ins, int64_t kh, int64_t kw) {
    if (ins.op != MdxOp::Conv || ins.groups != 1 || ins.dilation[0] != 1 || ins.dilation[1] != 1) return false;
    if (kh != kw || ins.stride[0] != ins.stride[1] || ins.padding[0] != ins.padding[1]) return false;
    const int s = ins.stride[0], p = ins.padding[0];
    return (kh == 1 && s == 1 && p == 0) || (kh == 3 && s == 1 && p == 1) || (kh == 2 && s == 2 && p == 0);
}

// The patch matrix's GEMM takes oh·ow as an int column count.
bool npos_fits(const MdxConvShape& c) { return (int64_t)c.oh * c.ow <= INT32_MAX; }

// ConvTranspose 2 × 2, stride 2, no padding or output padding, ungrouped and undilated: one
// GEMM over the input positions with rows (co, dy, dx), then a scatter (mdx_shuffle2x2).
bool gemm_transpose_geometry(const MdxInstruction& ins, int64_t kh, int64_t kw) {
    return ins.op == MdxOp::ConvTranspose && ins.groups == 1 && kh == 2 && kw == 2 && ins.stride[0] == 2 &&
           ins.stride[1] == 2 && ins.padding[0] == 0 && ins.padding[1] == 0 && ins.padding_out[0] == 0 &&
           ins.padding_out[1] == 0 && ins.dilation[0] == 1 && ins.dilation[1] == 1;
}

GemmEpilogue plain_f32_epilogue() {
    GemmEpilogue e{};
    e.act = ANCHA_ACT_NONE;
    e.out_type = ELT_F32;
    e.rope_tokens = 1;
    e.rope_div = 1;
    e.rope_hd = 64;
    return e;
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
    std::string err;
    if (!graph.infer(in, shapes, err)) return fail(ANCHA_E_INVALID, err);
    return ANCHA_OK;
}

int MdxModel::set_gemm(int precision) {
    if (precision < 0) {
        gemm_elt_ = -1;
        gemm_w_.clear();
        gemm_kp_.clear();
        return ANCHA_OK;
    }
    if (precision != ANCHA_PRECISION_F32 && precision != ANCHA_PRECISION_BF16 && precision != ANCHA_PRECISION_F16)
        return fail(ANCHA_E_INVALID, "mdx_set_gemm: unknown precision");
    const int elt = precision == ANCHA_PRECISION_BF16 ? ELT_BF16 : precision == ANCHA_PRECISION_F16 ? ELT_F16 : ELT_F32;
    ANCHA_CUDA(cudaSetDevice(device));
    const size_t n = graph.instructions.size();
    std::vector<DevBuf> w(n);
    std::vector<int64_t> kp(n, 0);
    try {
        for (size_t k = 0; k < n; ++k) {
            const MdxInstruction& ins = graph.instructions[k];
            if ((ins.op != MdxOp::Conv && ins.op != MdxOp::MatMul && ins.op != MdxOp::ConvTranspose) ||
                ins.inputs[1] >= (int)graph.constants.size())
                continue;
            const MdxConstant& wc = graph.constants[ins.inputs[1]];
            if (ins.op == MdxOp::ConvTranspose) {
                // [ci][co][2][2] (BatchNormalization folded in when optimized) as rows
                // (co, dy, dx) over ci, padded to kp.
                if (!gemm_transpose_geometry(ins, wc.shape[2], wc.shape[3])) continue;
                const int64_t ci = wc.shape[0], co = wc.shape[1], p = (ci + 7) / 8 * 8;
                std::vector<float> rows((size_t)(co * 4 * p), 0.f);
                for (int64_t i = 0; i < ci; ++i)
                    for (int64_t o = 0; o < co; ++o)
                        for (int64_t t = 0; t < 4; ++t)
                            rows[(size_t)((o * 4 + t) * p + i)] = wc.data[(size_t)((i * co + o) * 4 + t)];
                upload_elt(w[k], rows, elt);
                kp[k] = p;
                continue;
            }
            if (ins.op == MdxOp::MatMul) {
                // A constant 2-D right operand [K][N] for the tensor cores: its transpose [N][K]
                // (the NK operand) in the 16-bit type. f32 mode reads the constant as stored.
                const int64_t kk = wc.shape[2], nn = wc.shape[3];
                if (elt == ELT_F32 || wc.shape[0] != 1 || wc.shape[1] != 1 || kk % 8) continue;
                std::vector<float> t((size_t)(kk * nn));
                for (int64_t r = 0; r < kk; ++r)
                    for (int64_t c = 0; c < nn; ++c) t[(size_t)(c * kk + r)] = wc.data[(size_t)(r * nn + c)];
                upload_elt(w[k], t, elt);
                kp[k] = kk;
                continue;
            }
            if (!gemm_geometry(ins, wc.shape[2], wc.shape[3])) continue;
            // [co][ci][kh][kw] flattened is the patch order (c, ky, kx); rows padded to kp.
            const int64_t co = wc.shape[0], kk = wc.shape[1] * wc.shape[2] * wc.shape[3];
            const int64_t p = (kk + 7) / 8 * 8;
            std::vector<float> padded((size_t)(co * p), 0.f);
            for (int64_t o = 0; o < co; ++o)
                std::copy(wc.data.begin() + o * kk, wc.data.begin() + (o + 1) * kk, padded.begin() + o * p);
            upload_elt(w[k], padded, elt);
            kp[k] = p;
        }
    } catch (const std::exception& e) {
        return fail(ANCHA_E_CUDA, e.what());
    }
    gemm_w_ = std::move(w);
    gemm_kp_ = std::move(kp);
    gemm_elt_ = elt;
    return ANCHA_OK;
}

int MdxModel::conv_as_gemm(size_t k, const float* x, const float* bias, bool relu, float* y, const MdxConvShape& c,
                           cudaStream_t s) {
    const int64_t kp = gemm_kp_[k], npos = (int64_t)c.oh * c.ow;
    const size_t es = elt_size(gemm_elt_);
    if ((int64_t)c.ci * c.kh * c.kw > kp) return fail(ANCHA_E_INVALID, "mdx conv_gemm: weight / input channels");
    void* patches = nullptr;
    if (cudaMallocAsync(&patches, (size_t)c.n * npos * kp * es, s) != cudaSuccess)
        return fail(ANCHA_E_CUDA, "cudaMallocAsync of an MDX patch matrix");
    PackArgs p{};
    p.a = PackSource{x, c.ci, nullptr, nullptr, nullptr};  // no norm, no activation: plain im2col
    p.b = PackSource{nullptr, 0, nullptr, nullptr, nullptr};
    p.batch = c.n; p.h = c.h; p.w = c.w; p.ho_n = c.oh; p.wo_n = c.ow;
    p.kh = c.kh; p.kw = c.kw; p.sh = c.sh; p.sw = c.sw; p.ph = c.ph; p.pw = c.pw;
    p.gelu = false; p.eps = 0.f; p.kp = kp; p.out = patches; p.out_type = gemm_elt_;
    int st = mdx_pack(p, s);
    const GemmEpilogue e = plain_f32_epilogue();
    for (int i = 0; i < c.n && st == ANCHA_OK; ++i) {
        // Image i: y[i] [co][oh·ow] = W [co][kp] · P[i] [oh·ow][kp]ᵀ, NCHW as it stands.
        GemmGroup g{};
        g.a = gemm_w_[k].p; g.lda = kp;
        g.b = static_cast<const uint8_t*>(patches) + (size_t)i * npos * kp * es; g.ldb = kp;
        g.out = y + (size_t)i * c.co * npos; g.ldo = npos; g.ldr = npos;
        g.m = c.co; g.n = (int)npos; g.k = (int)kp;
        st = ANCHA_E_UNSUPPORTED;
        if (gemm_elt_ != ELT_F32) st = gemm_tc(g, gemm_elt_, e, s);
        if (st == ANCHA_E_UNSUPPORTED) st = gemm_ffma(g, nullptr, 1, g.m, g.n, gemm_elt_, gemm_elt_, 1, e, s);
    }
    cudaFreeAsync(patches, s);
    if (st == ANCHA_OK) st = mdx_channel_affine(y, nullptr, bias, y, c.n, c.co, npos, relu, s);
    return st;
}

int MdxModel::conv_transpose_as_gemm(size_t k, const float* x, const float* bias, bool relu, float* y,
                                     const MdxConvShape& c, cudaStream_t s) {
    const int64_t kp = gemm_kp_[k], npos = (int64_t)c.h * c.w;
    const size_t es = elt_size(gemm_elt_);
    if (c.ci > kp || c.oh != 2 * c.h || c.ow != 2 * c.w) return fail(ANCHA_E_INVALID, "mdx conv_gemm: transpose shape");
    void* patches = nullptr;
    float* raw = nullptr;
    if (cudaMallocAsync(&patches, (size_t)c.n * npos * kp * es, s) != cudaSuccess)
        return fail(ANCHA_E_CUDA, "cudaMallocAsync of an MDX patch matrix");
    if (cudaMallocAsync(reinterpret_cast<void**>(&raw), (size_t)c.n * c.co * 4 * npos * sizeof(float), s) != cudaSuccess) {
        cudaFreeAsync(patches, s);
        return fail(ANCHA_E_CUDA, "cudaMallocAsync of an MDX transposed-convolution product");
    }
    PackArgs p{};  // 1 × 1 gather: the input as [image][position][channel]
    p.a = PackSource{x, c.ci, nullptr, nullptr, nullptr};
    p.b = PackSource{nullptr, 0, nullptr, nullptr, nullptr};
    p.batch = c.n; p.h = c.h; p.w = c.w; p.ho_n = c.h; p.wo_n = c.w;
    p.kh = p.kw = 1; p.sh = p.sw = 1; p.ph = p.pw = 0;
    p.gelu = false; p.eps = 0.f; p.kp = kp; p.out = patches; p.out_type = gemm_elt_;
    int st = mdx_pack(p, s);
    const GemmEpilogue e = plain_f32_epilogue();
    for (int i = 0; i < c.n && st == ANCHA_OK; ++i) {
        // raw[i] [(co, dy, dx)][h·w] = W' [4·co][kp] · P[i] [h·w][kp]ᵀ
        GemmGroup g{};
        g.a = gemm_w_[k].p; g.lda = kp;
        g.b = static_cast<const uint8_t*>(patches) + (size_t)i * npos * kp * es; g.ldb = kp;
        g.out = raw + (size_t)i * c.co * 4 * npos; g.ldo = npos; g.ldr = npos;
        g.m = 4 * c.co; g.n = (int)npos; g.k = (int)kp;
        st = ANCHA_E_UNSUPPORTED;
        if (gemm_elt_ != ELT_F32) st = gemm_tc(g, gemm_elt_, e, s);
        if (st == ANCHA_E_UNSUPPORTED) st = gemm_ffma(g, nullptr, 1, g.m, g.n, gemm_elt_, gemm_elt_, 1, e, s);
    }
    if (st == ANCHA_OK) st = mdx_shuffle2x2(raw, c.n, c.co, c.h, c.w, y, c.co, 0, s);
    cudaFreeAsync(patches, s);
    cudaFreeAsync(raw, s);
    if (st == ANCHA_OK) st = mdx_channel_affine(y, nullptr, bias, y, c.n, c.co, 4 * npos, relu, s);
    return st;
}

int MdxModel::matmul_as_tc(size_t k, const float* a, int64_t rows, int kk, int nn, float* y, cudaStream_t s) {
    if (gemm_kp_[k] != kk) return fail(ANCHA_E_UNSUPPORTED, "mdx conv_gemm: no tensor-core weight");
    void* a16 = nullptr;
    if (cudaMallocAsync(&a16, (size_t)rows * kk * 2, s) != cudaSuccess)
        return fail(ANCHA_E_CUDA, "cudaMallocAsync of an MDX MatMul operand");
    int st = cast_rows(a, kk, a16, gemm_elt_, kk, rows, kk, s);
    GemmGroup g{};
    g.a = a16; g.lda = kk;
    g.b = gemm_w_[k].p; g.ldb = kk;
    g.out = y; g.ldo = nn; g.ldr = nn;
    g.m = (int)rows; g.n = nn; g.k = kk;
    if (st == ANCHA_OK) st = gemm_tc(g, gemm_elt_, plain_f32_epilogue(), s);
    cudaFreeAsync(a16, s);
    return st;
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
    // conv_gemm: a Relu that is the next instruction and the only consumer of a convolution run
    // as a GEMM, or of a BatchNormalization, is applied in that instruction's pass, and its value
    // is that instruction's buffer.
    auto relu_follows = [&](size_t k) {
        const MdxInstruction& ins = graph.instructions[k];
        return k + 1 < graph.instructions.size() && graph.instructions[k + 1].op == MdxOp::Relu &&
               graph.instructions[k + 1].inputs[0] == ins.output && graph.uses[ins.output] == 1;
    };
    int st = ANCHA_OK;
    for (size_t k = 0; k < graph.instructions.size() && st == ANCHA_OK; ++k) {
        if (cancel && *cancel) { st = fail(ANCHA_E_CANCELLED, "task cancelled"); break; }
        const MdxInstruction& ins = graph.instructions[k];
        bool relu_done = false;
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
                mdx_conv_shape(ins, a, shapes[ins.inputs[1]], c, err);  // checked by infer
                const float* bias = ins.inputs.size() == 3 ? values[ins.inputs[2]] : nullptr;
                st = ANCHA_E_UNSUPPORTED;
                if (gemm_elt_ >= 0 && gemm_kp_[k] && npos_fits(c)) {
                    const bool relu = relu_follows(k);
                    st = ins.op == MdxOp::Conv ? conv_as_gemm(k, va, bias, relu, y, c, s)
                                               : conv_transpose_as_gemm(k, va, bias, relu, y, c, s);
                    relu_done = relu && st == ANCHA_OK;
                }
                if (st == ANCHA_E_UNSUPPORTED)
                    st = mdx_conv2d(va, values[ins.inputs[1]], bias, y, c, ins.op == MdxOp::ConvTranspose, s);
                break;
            }
            case MdxOp::Relu:
            case MdxOp::Add:
            case MdxOp::Mul:
            case MdxOp::Bn: {
                if (ins.op == MdxOp::Bn && gemm_elt_ >= 0 && relu_follows(k)) {
                    // conv_gemm: the BatchNormalization and the Relu after it in one pass.
                    st = mdx_channel_affine(va, bn_scale_[k].as<float>(), bn_shift_[k].as<float>(), y, a[0], (int)a[1],
                                            a[2] * a[3], true, s);
                    relu_done = st == ANCHA_OK;
                    break;
                }
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
                const int64_t rows = a[0] * a[1] * a[2];
                if (gemm_elt_ >= 0 && ins.inputs[1] < nconst && b[0] == 1 && b[1] == 1 && rows <= 65535LL * 128) {
                    // [a0·a1·m, k] · [k, n] in one FFMA GEMM (right operand KN, as ONNX stores it).
                    // 16-bit modes: A cast once, then the tensor cores; f32 (or a shape the
                    // tensor-core kernel declines, with nothing written): the FFMA GEMM.
                    st = ANCHA_E_UNSUPPORTED;
                    if (gemm_elt_ != ELT_F32) st = matmul_as_tc(k, va, rows, (int)a[3], (int)b[3], y, s);
                    if (st == ANCHA_E_UNSUPPORTED) {
                        GemmGroup g{};
                        g.a = va; g.lda = a[3];
                        g.b = values[ins.inputs[1]]; g.ldb = b[3];
                        g.out = y; g.ldo = b[3]; g.ldr = b[3];
                        g.m = (int)rows; g.n = (int)b[3]; g.k = (int)a[3];
                        st = gemm_ffma(g, nullptr, 1, g.m, g.n, ELT_F32, ELT_F32, 0, plain_f32_epilogue(), s);
                    }
                    break;
                }
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
        if (relu_done) {  // the fused Relu (instruction k + 1): its value is this buffer
            values[graph.instructions[k + 1].output] = values[ins.output];
            values[ins.output] = nullptr;
            --uses[ins.output];
            ++k;
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

int MdxModel::separate_pcm(const MdxTaskOpts& o, const float* planes, int64_t samples, const volatile int* cancel,
                           float* predicted, float* residual, double* seconds) {
    const auto t0 = std::chrono::steady_clock::now();
    // separate_mdx (src/mdx_runtime.rs:84-248): option checks, UVR trim / pad, chunk starts.
    if (!planes || !predicted || !residual || samples <= 0) return fail(ANCHA_E_INVALID, "mdx_separate: empty input");
    if (samples > kMaxTrackSamples) return fail(ANCHA_E_INVALID, "mdx_separate: track longer than 2^36 samples");
    if (o.batch < 1 || o.batch > 4) return fail(ANCHA_E_INVALID, "MDX batch size must be between 1 and 4");
    if (std::isnan(o.overlap) || (o.overlap >= 0.0 && !(o.overlap <= 0.95)))
        return fail(ANCHA_E_INVALID, "MDX overlap must be between 0 and 0.95");
    if (o.hop <= 0 || o.hop > o.n_fft || o.frames < 2 || o.bins <= 0 || o.bins > o.n_fft / 2 + 1)
        return fail(ANCHA_E_INVALID, "invalid MDX STFT configuration");
    if (!mdx_task_fft_supported(o.n_fft)) return fail(ANCHA_E_UNSUPPORTED, "classic MDX STFT size not supported");
    const int64_t chunk = (int64_t)o.hop * (o.frames - 1);  // < 2^62: no overflow
    if (chunk > kMaxChunkSamples) return fail(ANCHA_E_INVALID, "MDX chunk longer than 60 s");
    const int64_t trim = o.n_fft / 2, gen = chunk - o.n_fft;
    if (gen <= 0 || chunk <= trim) return fail(ANCHA_E_INVALID, "MDX chunk shorter than its FFT");
    const int64_t pad = gen + trim - samples % gen;
    const int64_t mixture = trim + samples + pad;
    const int64_t step = o.overlap < 0.0 ? gen : (int64_t)((1.0 - o.overlap) * (double)chunk);
    if (step <= 0) return fail(ANCHA_E_INVALID, "zero MDX step");
    std::vector<int64_t> starts;
    for (int64_t s0 = 0; s0 < mixture; s0 += step)
        if (s0 < trim + samples) starts.push_back(s0);  // chunks past the track are skipped (optimized)
    ANCHA_CUDA(cudaSetDevice(device));
    const int b = o.batch, bins = o.bins, frames = o.frames, n = o.n_fft;
    const Shape4 in{b, 4, bins, frames};
    Shape4 out_shape{};
    ANCHA_TRY(output_shape(in, out_shape));
    if (out_shape != in) return fail(ANCHA_E_INVALID, "MDX output shape mismatch");
    try {
        DevBuf track, audio, spec, neg, y, y2, scratch, waves, result, divisor, pred, res, win, tw, flag;
        cudaStream_t s = nullptr;
        ANCHA_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
        struct StreamGuard {  // destroyed before the buffers (declared after them)
            cudaStream_t s;
            ~StreamGuard() {
                cudaStreamSynchronize(s);
                cudaStreamDestroy(s);
            }
        } guard{s};
        const size_t spec_n = (size_t)b * 4 * bins * frames;
        track.alloc((size_t)2 * samples * 4);
        audio.alloc((size_t)b * 2 * chunk * 4);
        spec.alloc(spec_n * 4);
        y.alloc(spec_n * 4);
        if (o.denoise) {
            neg.alloc(spec_n * 4);
            y2.alloc(spec_n * 4);
        }
        scratch.alloc((size_t)b * 2 * frames * n * 4);
        waves.alloc((size_t)b * 2 * chunk * 4);
        result.alloc((size_t)2 * samples * 4);
        divisor.alloc((size_t)samples * 4);
        pred.alloc((size_t)2 * samples * 4);
        res.alloc((size_t)2 * samples * 4);
        win.alloc((size_t)n * 4);
        tw.alloc((size_t)(n / 2 + 1) * sizeof(float2));
        flag.alloc(sizeof(int));
        ANCHA_CUDA(cudaMemcpyAsync(track.p, planes, (size_t)2 * samples * 4, cudaMemcpyHostToDevice, s));
        ANCHA_CUDA(cudaMemsetAsync(result.p, 0, result.bytes, s));
        ANCHA_CUDA(cudaMemsetAsync(divisor.p, 0, divisor.bytes, s));
        ANCHA_CUDA(cudaMemsetAsync(flag.p, 0, sizeof(int), s));
        ANCHA_TRY(mdx_task_tables(n, win.as<float>(), tw.as<float2>(), s));
        for (size_t i = 0; i < starts.size(); i += b) {
            if (cancel && *cancel) return fail(ANCHA_E_CANCELLED, "task cancelled");
            const int cnt = (int)std::min<size_t>(b, starts.size() - i);
            MdxChunks4 ch{};
            for (int c = 0; c < cnt; ++c) {
                ch.start[c] = starts[i + c];
                ch.actual[c] = std::min<int64_t>(chunk, mixture - starts[i + c]);
            }
            ANCHA_TRY(mdx_task_gather(track.as<float>(), samples, ch, cnt, (int)chunk, trim, audio.as<float>(), s));
            if (cnt < b) ANCHA_CUDA(cudaMemsetAsync(spec.as<float>() + (size_t)cnt * 4 * bins * frames, 0,
                                                    (size_t)(b - cnt) * 4 * bins * frames * 4, s));
            ANCHA_TRY(mdx_task_stft(audio.as<float>(), cnt, (int)chunk, o.hop, n, bins, 3, win.as<float>(),
                                    tw.as<float2>(), spec.as<float>(), s));
            // The graph runs on the batch it was shaped for; unused slots hold zeros.
            if (o.denoise) {
                ANCHA_TRY(mdx_negate(spec.as<float>(), (int64_t)spec_n, neg.as<float>(), s));
                ANCHA_TRY(forward(neg.as<float>(), in, y2.as<float>(), cancel, s));
                ANCHA_TRY(forward(spec.as<float>(), in, y.as<float>(), cancel, s));
                ANCHA_TRY(mdx_half_difference(y.as<float>(), y2.as<float>(), (int64_t)spec_n, y.as<float>(), s));
            } else {
                ANCHA_TRY(forward(spec.as<float>(), in, y.as<float>(), cancel, s));
            }
            ANCHA_TRY(mdx_task_istft(y.as<float>(), cnt, bins, frames, o.hop, (int)chunk, n, win.as<float>(),
                                     tw.as<float2>(), scratch.as<float>(), waves.as<float>(), flag.as<int>(), s));
            ANCHA_TRY(mdx_task_ola(waves.as<float>(), ch, cnt, (int)chunk, trim, samples, o.overlap == 0.0,
                                   result.as<float>(), divisor.as<float>(), s));
        }
        ANCHA_TRY(mdx_task_finish(result.as<float>(), divisor.as<float>(), track.as<float>(), samples, o.compensate,
                                  pred.as<float>(), res.as<float>(), flag.as<int>(), s));
        ANCHA_CUDA(cudaMemcpyAsync(predicted, pred.p, pred.bytes, cudaMemcpyDeviceToHost, s));
        ANCHA_CUDA(cudaMemcpyAsync(residual, res.p, res.bytes, cudaMemcpyDeviceToHost, s));
        int status = 0;
        ANCHA_CUDA(cudaMemcpyAsync(&status, flag.p, sizeof(int), cudaMemcpyDeviceToHost, s));
        ANCHA_CUDA(cudaStreamSynchronize(s));
        if (status & 1) return fail(ANCHA_E_NONFINITE, "non-finite MDX output");
        if (status & 2) return fail(ANCHA_E_INVALID, "MDX OLA uncovered sample; overlap setting is invalid");
    } catch (const std::exception& e) {
        return fail(ANCHA_E_CUDA, e.what());
    }
    if (seconds) *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    return ANCHA_OK;
}

}  // namespace ancha
