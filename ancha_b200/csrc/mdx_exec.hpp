// Classic MDX graph executor on the device: the schedule of onnx.hpp's MdxGraph run over 4-D
// f32 NCHW tensors (Graph::forward, crates/ancha-models/src/mdx.rs:474-568). Shapes are
// inferred on the host before any launch; intermediate values live in stream-ordered
// allocations released when their last consumer has run.
#pragma once
#include <array>
#include <memory>
#include <vector>

#include "common.cuh"
#include "model.hpp"
#include "onnx.hpp"

namespace ancha {

struct MdxConvShape {
    int n, ci, h, w, co, oh, ow, kh, kw, sh, sw, ph, pw, dh, dw, groups;
};
// Elementwise op (0 Relu, 1 Add, 2 Mul, 3 per-channel x·scale + shift) over a 4-D output;
// sa / sb are the inputs' element strides, 0 on broadcast dims (for op 3, sb indexes scale /
// shift by channel).
struct MdxEwise {
    int op;
    int64_t out[4], sa[4], sb[4];
    const float* scale;
    const float* shift;
};
struct MdxPermute {
    int64_t out[4], stride[4];  // stride: input element stride of each output dim
};
// Batched [m × k]·[k × n] over two broadcast batch dims (sa / sb: batch strides, 0 when
// broadcast); the output is contiguous [batch0][batch1][m][n].
struct MdxMatmul {
    int64_t batch[2], sa[2], sb[2];
    int m, n, k;
};

int mdx_conv2d(const float* x, const float* w, const float* bias, float* out, const MdxConvShape& c, bool transpose,
               cudaStream_t s);
int mdx_ewise(const float* a, const float* b, float* out, const MdxEwise& e, cudaStream_t s);
int mdx_permute(const float* x, float* out, const MdxPermute& p, cudaStream_t s);
int mdx_matmul(const float* a, const float* b, float* out, const MdxMatmul& m, cudaStream_t s);

using Shape4 = std::array<int64_t, 4>;

class MdxModel {
public:
    // Reads and validates the ONNX model (MdxGraph::build) and uploads its constants.
    static std::unique_ptr<MdxModel> load(const uint8_t* onnx, size_t bytes, bool optimized, int device);
    // Output shape for an input shape; ANCHA_E_INVALID when an op's shapes disagree.
    int output_shape(const Shape4& in, Shape4& out) const;
    // x: device [in] f32 → out: device, of output_shape(in). Checks *cancel (host, may be
    // null) before every instruction (mdx.rs:484).
    int forward(const float* x, const Shape4& in, float* out, const volatile int* cancel, cudaStream_t s);

    MdxGraph graph;
    int device = 0;

private:
    int infer(const Shape4& in, std::vector<Shape4>& shapes) const;
    std::vector<DevBuf> constants_;          // by value id
    std::vector<DevBuf> bn_scale_, bn_shift_;  // by instruction (BatchNormalization only)
};

}  // namespace ancha

struct ancha_mdx {
    std::unique_ptr<ancha::MdxModel> impl;
};
