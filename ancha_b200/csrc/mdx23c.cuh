// Device kernels of the MDX23C (TFC-TDF v3) network: per-plane instance-norm statistics,
// the fused norm → GELU → patch gather that feeds every convolution's GEMM, the row-wise
// norm → GELU that feeds the TDF GEMMs, plane transposes and the 2 × 2 transpose-convolution
// scatter. Activations are NCHW f32 planes; GEMM operands are f32, f16 or bf16.
#pragma once
#include "common.cuh"

namespace ancha {

// Sums and sums of squares (f64) of each contiguous plane of `n` floats, accumulated into
// `stats[plane]` (zeroed here first). The consumers derive mean and 1/sqrt(var + eps).
int mdx_plane_stats(const float* x, int64_t planes, int64_t n, double2* stats, cudaStream_t s);

// One NCHW source of a patch gather: `channels` planes of [h][w] per batch item, optional
// instance norm (stats from mdx_plane_stats over the same planes, gamma / beta per channel).
struct PackSource {
    const float* x;
    int channels;
    const double2* stats;  // [batch][channels] or null (no norm)
    const float* gamma;
    const float* beta;
};

// Patch matrix of a bias-free convolution: P[b][ho·wo_n + wo][k], k = (c·kh + ky)·kw + kx
// over the channels of `a` then `b` (a channel concatenation), value = act(norm(x)) at input
// (ho·sh − ph + ky, wo·sw − pw + kx) or 0 outside the plane; columns K..kp−1 are 0. `gelu`
// applies the exact erf GELU after the norm. P is of element type `out_type`.
struct PackArgs {
    PackSource a, b;
    int batch, h, w, ho_n, wo_n;
    int kh, kw, sh, sw, ph, pw;
    bool gelu;
    float eps;
    int64_t kp;
    void* out;
    int out_type;
};
int mdx_pack(const PackArgs& a, cudaStream_t s);

// out[i] = act(norm(x[i])) over `planes` contiguous planes of `n` floats (plane index
// i / n, channel (i / n) % channels), written as `out_type`; the TDF GEMM input.
int mdx_norm_act(const float* x, int64_t planes, int64_t n, int channels, const double2* stats,
                 const float* gamma, const float* beta, float eps, bool gelu, void* out,
                 int out_type, cudaStream_t s);

// out[p][c][r] = x[p][r][c] · (mul ? mul[p][c][r] : 1) for `planes` planes of rows × cols.
int mdx_transpose(const float* x, const float* mul, int64_t planes, int rows, int cols, float* out,
                  cudaStream_t s);

// Scatter of the 2 × 2, stride-2 transpose convolution's GEMM output y[b][(c·2 + dy)·2 + dx]
// [h·w + x] into out[b][c_off + c][2·h + dy][2·x + dx] (out holds c_total channels).
int mdx_shuffle2x2(const float* y, int batch, int channels, int h, int w, float* out, int c_total,
                   int c_off, cudaStream_t s);

}  // namespace ancha
