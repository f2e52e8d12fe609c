// Classic MDX graph executor on the device: the schedule of onnx.hpp's MdxGraph run over 4-D
// f32 NCHW tensors (Graph::forward, crates/ancha-models/src/mdx.rs:474-568). Shapes are
// inferred on the host before any launch; intermediate values live in stream-ordered
// allocations released when their last consumer has run.
#pragma once
#include <array>
#include <memory>
#include <vector>

#include "common.cuh"
#include "mdx23c.cuh"
#include "model.hpp"
#include "onnx.hpp"

namespace ancha {

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
// y[i][c][·] = x[i][c][·] · scale[c] + shift[c] (scale / shift may be null: 1 / 0), then
// max(·, 0) when `relu`, for `batch` images of `channels` planes of `plane` elements; x may be
// y. Serves the bias (and a following Relu) of a convolution run as a GEMM, whose epilogue bias
// runs along the other axis, and a BatchNormalization with the Relu that follows it.
int mdx_channel_affine(const float* x, const float* scale, const float* shift, float* y, int64_t batch, int channels,
                       int64_t plane, bool relu, cudaStream_t s);

// ---- The classic MDX task (src/mdx_runtime.rs) -------------------------------------------------

// Up to four chunks of one batch: start in the trimmed / padded mixture and valid length.
struct MdxChunks4 {
    int64_t start[4];
    int64_t actual[4];
};
// True when the task's STFT can run n_fft points: n_fft/2 = 2^k, 3·2^k or 5·2^k, n_fft ≤ 8192.
bool mdx_task_fft_supported(int n_fft);
// Periodic Hann window [n_fft] (f32 form of dsp.rs:40-42) and exp(−2πij/n_fft), j ≤ n_fft/2.
int mdx_task_tables(int n_fft, float* window, float2* twiddle, cudaStream_t s);
// Centred STFT of audio[c][2][samples] packed as [c][4][bins][frames] with bins < zero_low
// zeroed (mdx_runtime.rs:79-83).
int mdx_task_stft(const float* audio, int chunks, int samples, int hop, int n_fft, int bins, int zero_low,
                  const float* window, const float2* twiddle, float* packed, cudaStream_t s);
// Inverse of spec[c][4][bins][frames] (spectral::unpack + Stft::inverse) into waves[c][2][samples];
// scratch holds chunks·2·frames·n_fft floats.
int mdx_task_istft(const float* spec, int chunks, int bins, int frames, int hop, int samples, int n_fft,
                   const float* window, const float2* twiddle, float* scratch, float* waves, int* flag, cudaStream_t s);
// Chunk windows of the mixture: out[c][ch][i] = planes[ch][start + i − trim] for i < actual inside
// the track, else 0 (mdx_runtime.rs:152-169).
int mdx_task_gather(const float* planes, int64_t samples, const MdxChunks4& ch, int chunks, int chunk, int64_t trim,
                    float* out, cudaStream_t s);
// Hann-weighted (or rectangular) overlap-add of waves[c][2][chunk] into result[2][samples] and
// divisor[samples], chunks in order (mdx_runtime.rs:205-224).
int mdx_task_ola(const float* waves, const MdxChunks4& ch, int chunks, int chunk, int64_t trim, int64_t samples,
                 bool rectangular, float* result, float* divisor, cudaStream_t s);
// predicted = result / divisor · compensate, residual = input − predicted (mdx_runtime.rs:227-237).
int mdx_task_finish(const float* result, const float* divisor, const float* input, int64_t samples, float compensate,
                    float* predicted, float* residual, int* flag, cudaStream_t s);
int mdx_negate(const float* a, int64_t n, float* out, cudaStream_t s);
int mdx_half_difference(const float* a, const float* b, int64_t n, float* out, cudaStream_t s);

// Options of the task (the MdxConfig fields of a registered checkpoint, given explicitly here).
struct MdxTaskOpts {
    int n_fft = 6144, hop = 1024, bins = 3072, frames = 256;
    float compensate = 1.f;
    double overlap = -1.0;  // < 0: chunks every chunk − n_fft samples (the reference's default)
    bool denoise = false;
    int batch = 1;          // chunks per graph call, 1..4
};

class MdxModel {
public:
    // Reads and validates the ONNX model (MdxGraph::build) and uploads its constants.
    static std::unique_ptr<MdxModel> load(const uint8_t* onnx, size_t bytes, bool optimized, int device);
    // Output shape for an input shape; ANCHA_E_INVALID when an op's shapes disagree.
    int output_shape(const Shape4& in, Shape4& out) const;
    // x: device [in] f32 → out: device, of output_shape(in). Checks *cancel (host, may be
    // null) before every instruction (mdx.rs:484).
    int forward(const float* x, const Shape4& in, float* out, const volatile int* cancel, cudaStream_t s);
    // separate_mdx without file I/O (src/mdx_runtime.rs:84-248): host planes[2][samples] →
    // host predicted[2][samples] and residual[2][samples]; *seconds (may be null) = wall time.
    int separate_pcm(const MdxTaskOpts& o, const float* planes, int64_t samples, const volatile int* cancel,
                     float* predicted, float* residual, double* seconds);

    // Graph::forward's conv_gemm (mdx.rs:472-530, spatial.rs:21-67): ungrouped, undilated
    // convolutions with constant weights in the patch-gather geometries (1×1, 3×3 with padding
    // 1, 2×2 with stride 2) run as the weight matrix [co][ci·kh·kw] times a patch matrix, 2×2 /
    // stride-2 ConvTranspose layers as a GEMM with rows (co, dy, dx) plus a scatter (as the
    // MDX23C decoder does), and a MatMul by a constant 2-D right operand as one GEMM. precision < 0: off, every op on
    // its direct kernel (the default). ANCHA_PRECISION_F32: those GEMMs on the FFMA kernel.
    // ANCHA_PRECISION_BF16 / _F16: on the tcgen05 kernel with 16-bit weights and operands
    // (patches; MatMul inputs cast once), fp32 accumulation and output. Uploads the converted
    // weights; not re-entrant with forward on the same handle.
    int set_gemm(int precision);

    MdxGraph graph;
    int device = 0;

private:
    int infer(const Shape4& in, std::vector<Shape4>& shapes) const;
    // Instruction k (an eligible Conv) on x as pack + GEMM + bias into y; ANCHA_E_UNSUPPORTED,
    // with nothing enqueued, when the patch gather does not take the shape.
    // `relu`: apply the Relu that follows in the same pass.
    int conv_as_gemm(size_t k, const float* x, const float* bias, bool relu, float* y, const MdxConvShape& c,
                     cudaStream_t s);
    // Instruction k (an eligible 2 × 2 / stride-2 ConvTranspose) as 1 × 1 gather + GEMM with rows
    // (co, dy, dx) + scatter + bias into y; ANCHA_E_UNSUPPORTED as above.
    int conv_transpose_as_gemm(size_t k, const float* x, const float* bias, bool relu, float* y,
                               const MdxConvShape& c, cudaStream_t s);
    // Instruction k (a MatMul by a constant [K][N]) on rows × K inputs a as cast + tcgen05 GEMM
    // into y; ANCHA_E_UNSUPPORTED, with nothing written to y, when the GEMM declines the shape.
    int matmul_as_tc(size_t k, const float* a, int64_t rows, int kk, int nn, float* y, cudaStream_t s);
    int gemm_elt_ = -1;             // ELT_* of the GEMMs, −1 = off
    // by instruction, in gemm_elt_: Conv [co][kp], ConvTranspose [(co, dy, dx)][kp], MatMul [N][K]
    std::vector<DevBuf> gemm_w_;
    std::vector<int64_t> gemm_kp_;  // by instruction: kp (ci·kh·kw or ci, rounded up to 8), MatMul K; 0 = none
    std::vector<DevBuf> constants_;          // by value id
    std::vector<DevBuf> bn_scale_, bn_shift_;  // by instruction (BatchNormalization only)
};

}  // namespace ancha

struct ancha_mdx {
    std::unique_ptr<ancha::MdxModel> impl;
};
