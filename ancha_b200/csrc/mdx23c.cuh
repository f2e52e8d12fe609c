// Device kernels of the MDX23C (TFC-TDF v3) network: per-plane instance-norm statistics,
// the fused norm → GELU → patch gather that feeds every convolution's GEMM, the row-wise
// norm → GELU that feeds the TDF GEMMs, plane transposes and the 2 × 2 transpose-convolution
// scatter. Activations are NCHW f32 planes; GEMM operands are f32, f16 or bf16.
#pragma once
#include "common.cuh"

namespace ancha {

// Adds Σ x and Σ x² (f64) of each of `planes` contiguous planes of `n` floats into
// sums[plane] (which the caller zeroes): the statistics of a tensor that no GEMM epilogue
// produced (the GEMMs accumulate theirs, GemmEpilogue::stats).
int mdx_plane_sums(const float* x, int64_t planes, int64_t n, double2* sums, cudaStream_t s);

// One NCHW source of a gather: `channels` planes of [h][w] per batch item and, when `sums` is
// set, their instance norm γ[c]·(x − mean)/√(var + eps) + β[c] from the planes' (Σ x, Σ x²)
// (biased variance, mdx23c.rs:200-213); gamma / beta start at this source's first channel.
struct PackSource {
    const float* x;
    int channels;
    const double2* sums;  // [batch · channels] or null (no norm)
    const float* gamma;
    const float* beta;
};

// Patch matrix of a bias-free convolution: P[b][ho·wo_n + wo][k], k = (c·kh + ky)·kw + kx
// over the channels of `a` then `b` (a channel concatenation), value = act(norm(x)) at input
// (ho·sh − ph + ky, wo·sw − pw + kx) or 0 outside the plane; columns K..kp−1 are 0. `gelu`
// applies the exact erf GELU after the norm. P is of element type `out_type`. Geometries:
// 1×1 / stride 1, 3×3 / stride 1 and 2×2 / stride 2 (the network's three); kp % 8 == 0.
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

// Channels-last copy for the implicit-GEMM convolution: out[b][pos][c] (f16 / bf16) =
// act(norm(x)) over the channel concatenation of `a` and `b` (NCHW planes of `pos` values);
// a.channels + b.channels must be a multiple of 64.
int mdx_preact_nhwc(const PackSource& a, const PackSource& b, int batch, int64_t pos, bool gelu, float eps,
                    void* out, int out_type, cudaStream_t s);

// out[i] = act(norm(x[i])) over `planes` contiguous planes of `n` floats (plane p = i / n,
// channel p % channels, statistics sums[p]), written as `out_type`; the TDF GEMM input.
int mdx_norm_act(const float* x, int64_t planes, int64_t n, int channels, const double2* sums, const float* gamma,
                 const float* beta, float eps, bool gelu, void* out, int out_type, cudaStream_t s);

// out[p][c][r] = x[p][r][c] · (mul ? mul[p][c][r] : 1) for `planes` planes of rows × cols.
int mdx_transpose(const float* x, const float* mul, int64_t planes, int rows, int cols, float* out,
                  cudaStream_t s);

// Scatter of the 2 × 2, stride-2 transpose convolution's GEMM output y[b][(c·2 + dy)·2 + dx]
// [h·w + x] into out[b][c_off + c][2·h + dy][2·x + dx] (out holds c_total channels).
int mdx_shuffle2x2(const float* y, int batch, int channels, int h, int w, float* out, int c_total,
                   int c_off, cudaStream_t s);

// ---- Spectral runtime of the MDX23C task (src/mdx23c_runtime.rs, src/spectral.rs) ----------

// Per-device tables for an n_fft-point transform (n_fft a power of two, 32..8192): the
// periodic Hann window in the reference's f32 form and exp(−2πik/8192), k ≤ 4096, from which
// every smaller power-of-two twiddle is a strided read.
struct MdxDsp {
    int n_fft = 0;
    float* window = nullptr;   // [n_fft]
    float2* twiddle = nullptr; // [4097]
};
int mdx_dsp_tables(int n_fft, float* window, float2* twiddle, cudaStream_t s);

// UVR chunk windows of the zero-bordered track (mdx23c_runtime.rs:116-132):
// out[c][ch][i] = planes[ch][starts[c] + i − border] inside the track, else 0 (at most 4
// chunks per call, starts on the host).
int mdx_gather(const float* planes, int64_t samples, const int64_t* starts, int chunks, int chunk, int64_t border,
               float* out, cudaStream_t s);

// Centred periodic-Hann STFT (reflect padding inside each chunk, dsp.rs:52-79) packed as
// spectral::pack does (spectral.rs:5-36): audio[c][2][samples] → out[c][4][bins][frames]
// (L.re, L.im, R.re, R.im), frames = samples / hop + 1.
int mdx_stft(const MdxDsp& d, const float* audio, int chunks, int samples, int hop, int bins, float* out,
             cudaStream_t s);

// Inverse of each stem's packed spectrum (spectral::unpack + Stft::inverse, spectral.rs:38-76,
// dsp.rs:82-133; bins past `bins` are zero, Im of DC / Nyquist dropped, 1/n scale,
// window-square normalised overlap-add): spec[c][stems·4][bins][frames] →
// waves[c][stem][2][samples]. `scratch` holds chunks·stems·2·frames·n_fft floats; bit 2 of
// *flag is set where a sample is uncovered.
int mdx_istft(const MdxDsp& d, const float* spec, int chunks, int stems, int bins, int frames, int hop, int samples,
              float* scratch, float* waves, int* flag, cudaStream_t s);

// Window-square normalised overlap-add of windowed time frames scratch[plane][frame][n_fft]
// (any n_fft; `window` its periodic Hann) into out[plane][samples] (dsp.rs:82-133); bit 2 of
// *flag marks an uncovered sample.
int mdx_istft_overlap(const float* scratch, int64_t planes, int frames, int hop, int samples, int n_fft,
                      const float* window, float* out, int* flag, cudaStream_t s);

// Rectangular overlap-add of chunk outputs, in chunk order (mdx23c_runtime.rs:214-223):
// sums[p][j − border] += waves[c][p][j − starts[c]] for j in
// [max(start, border), min(start + chunk, border + samples)), p over stems·2 planes; at most
// 4 chunks per call (starts on the host, ascending). Bit 0 of *flag marks a non-finite value.
int mdx_overlap_add(const float* waves, const int64_t* starts, int chunks, int planes, int chunk, int64_t border,
                    int64_t samples, float* sums, int* flag, cudaStream_t s);

// x[i] *= k for i < n (the overlap-add's division by the overlap count).
int mdx_scale(float* x, int64_t n, float k, cudaStream_t s);

}  // namespace ancha
