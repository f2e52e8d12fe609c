// Device kernels of the classic MDX graph executor (mdx_exec.hpp): the op set of
// crates/ancha-models/src/mdx.rs (Graph::forward, mdx.rs:474-568) on 4-D f32 NCHW tensors.
// Convolutions here are direct FFMA loops with every ONNX parameter (stride, padding,
// dilation, groups, output padding); elementwise ops broadcast like numpy over four dims.
#include "mdx_exec.hpp"

namespace ancha {
namespace {

constexpr int kThreads = 256;

unsigned blocks_for(int64_t n) { return (unsigned)std::min<int64_t>(ceil_div(n, kThreads), 148 * 32); }

// out[b][o][y][x] = bias[o] + Σ_{c, ky, kx} x[b][g·cig + c][y·s − p + ky·d][x·s − p + kx·d] · w[o][c][ky][kx]
__global__ void conv2d_kernel(const float* __restrict__ x, const float* __restrict__ w,
                              const float* __restrict__ bias, float* __restrict__ out, MdxConvShape c) {
    const int64_t total = (int64_t)c.n * c.co * c.oh * c.ow;
    const int cig = c.ci / c.groups, cog = c.co / c.groups;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int ox = (int)(i % c.ow);
        const int oy = (int)((i / c.ow) % c.oh);
        const int o = (int)((i / ((int64_t)c.ow * c.oh)) % c.co);
        const int64_t b = i / ((int64_t)c.ow * c.oh * c.co);
        const int g = o / cog;
        float acc = bias ? bias[o] : 0.f;
        for (int ci = 0; ci < cig; ++ci) {
            const float* xp = x + ((b * c.ci + g * cig + ci) * (int64_t)c.h) * c.w;
            const float* wp = w + ((int64_t)o * cig + ci) * c.kh * c.kw;
            for (int ky = 0; ky < c.kh; ++ky) {
                const int iy = oy * c.sh - c.ph + ky * c.dh;
                if (iy < 0 || iy >= c.h) continue;
                for (int kx = 0; kx < c.kw; ++kx) {
                    const int ix = ox * c.sw - c.pw + kx * c.dw;
                    if (ix < 0 || ix >= c.w) continue;
                    acc = fmaf(xp[(int64_t)iy * c.w + ix], wp[ky * c.kw + kx], acc);
                }
            }
        }
        out[i] = acc;
    }
}

// Transposed convolution as a gather: output (Y, X) receives input (i, j) through tap
// (ky, kx) when Y = i·s − p + ky·d (and likewise X); weights w[ci][co / groups][kh][kw].
__global__ void conv_transpose2d_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                        const float* __restrict__ bias, float* __restrict__ out, MdxConvShape c) {
    const int64_t total = (int64_t)c.n * c.co * c.oh * c.ow;
    const int cig = c.ci / c.groups, cog = c.co / c.groups;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int ox = (int)(i % c.ow);
        const int oy = (int)((i / c.ow) % c.oh);
        const int o = (int)((i / ((int64_t)c.ow * c.oh)) % c.co);
        const int64_t b = i / ((int64_t)c.ow * c.oh * c.co);
        const int g = o / cog, ol = o % cog;
        float acc = bias ? bias[o] : 0.f;
        for (int ky = 0; ky < c.kh; ++ky) {
            const int ty = oy + c.ph - ky * c.dh;
            if (ty < 0 || ty % c.sh) continue;
            const int iy = ty / c.sh;
            if (iy >= c.h) continue;
            for (int kx = 0; kx < c.kw; ++kx) {
                const int tx = ox + c.pw - kx * c.dw;
                if (tx < 0 || tx % c.sw) continue;
                const int ix = tx / c.sw;
                if (ix >= c.w) continue;
                for (int ci = 0; ci < cig; ++ci) {
                    const int cc = g * cig + ci;
                    acc = fmaf(x[((b * c.ci + cc) * (int64_t)c.h + iy) * c.w + ix],
                               w[(((int64_t)cc * cog + ol) * c.kh + ky) * c.kw + kx], acc);
                }
            }
        }
        out[i] = acc;
    }
}

// Elementwise op over a 4-D output; each input is read through strides that are 0 on its
// broadcast dims.
__global__ void ewise_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ out,
                             MdxEwise e) {
    const int64_t total = e.out[0] * e.out[1] * e.out[2] * e.out[3];
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i, ia = 0, ib = 0;
        for (int d = 3; d >= 0; --d) {
            const int64_t k = r % e.out[d];
            r /= e.out[d];
            ia += k * e.sa[d];
            ib += k * e.sb[d];
        }
        const float va = a[ia];
        float v;
        if (e.op == 0) v = fmaxf(va, 0.f);
        else if (e.op == 1) v = va + b[ib];
        else if (e.op == 2) v = va * b[ib];
        else v = fmaf(va, e.scale[ib], e.shift[ib]);  // per-channel affine: b strides index the channel
        out[i] = v;
    }
}

__global__ void permute_kernel(const float* __restrict__ x, float* __restrict__ out, MdxPermute p) {
    const int64_t total = p.out[0] * p.out[1] * p.out[2] * p.out[3];
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i, src = 0;
        for (int d = 3; d >= 0; --d) {
            const int64_t k = r % p.out[d];
            r /= p.out[d];
            src += k * p.stride[d];
        }
        out[i] = x[src];
    }
}

// out[b0][b1] = a[b0 or 0][b1 or 0] · w[b0 or 0][b1 or 0] (16 × 16 shared-memory tiles).
__global__ void matmul_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ out,
                              MdxMatmul m) {
    __shared__ float ta[16][17], tb[16][17];
    const int64_t bz = blockIdx.z;
    const int64_t b0 = bz / m.batch[1], b1 = bz % m.batch[1];
    const float* A = a + b0 * m.sa[0] + b1 * m.sa[1];
    const float* B = b + b0 * m.sb[0] + b1 * m.sb[1];
    float* O = out + bz * (int64_t)m.m * m.n;
    const int row = blockIdx.y * 16 + threadIdx.y, col = blockIdx.x * 16 + threadIdx.x;
    float acc = 0.f;
    for (int k0 = 0; k0 < m.k; k0 += 16) {
        const int ka = k0 + threadIdx.x, kb = k0 + threadIdx.y;
        ta[threadIdx.y][threadIdx.x] = row < m.m && ka < m.k ? A[(int64_t)row * m.k + ka] : 0.f;
        tb[threadIdx.y][threadIdx.x] = kb < m.k && col < m.n ? B[(int64_t)kb * m.n + col] : 0.f;
        __syncthreads();
#pragma unroll
        for (int t = 0; t < 16; ++t) acc = fmaf(ta[threadIdx.y][t], tb[t][threadIdx.x], acc);
        __syncthreads();
    }
    if (row < m.m && col < m.n) O[(int64_t)row * m.n + col] = acc;
}

}  // namespace

int mdx_conv2d(const float* x, const float* w, const float* bias, float* out, const MdxConvShape& c, bool transpose,
               cudaStream_t s) {
    const int64_t total = (int64_t)c.n * c.co * c.oh * c.ow;
    if (total <= 0) return ANCHA_OK;
    if (transpose) conv_transpose2d_kernel<<<blocks_for(total), kThreads, 0, s>>>(x, w, bias, out, c);
    else conv2d_kernel<<<blocks_for(total), kThreads, 0, s>>>(x, w, bias, out, c);
    return check_launch(transpose ? "mdx_conv_transpose2d" : "mdx_conv2d");
}

int mdx_ewise(const float* a, const float* b, float* out, const MdxEwise& e, cudaStream_t s) {
    const int64_t total = e.out[0] * e.out[1] * e.out[2] * e.out[3];
    if (total <= 0) return ANCHA_OK;
    ewise_kernel<<<blocks_for(total), kThreads, 0, s>>>(a, b, out, e);
    return check_launch("mdx_ewise");
}

int mdx_permute(const float* x, float* out, const MdxPermute& p, cudaStream_t s) {
    const int64_t total = p.out[0] * p.out[1] * p.out[2] * p.out[3];
    if (total <= 0) return ANCHA_OK;
    permute_kernel<<<blocks_for(total), kThreads, 0, s>>>(x, out, p);
    return check_launch("mdx_permute");
}

namespace {
// x and y may alias (each element is read, then written, by one thread): no __restrict__.
__global__ void channel_affine_kernel(const float* x, const float* scale, const float* shift, float* y, int channels,
                                      int64_t plane, int64_t total, bool relu) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)((i / plane) % channels);
        float v = x[i];
        if (scale) v *= scale[c];
        if (shift) v += shift[c];
        y[i] = relu ? fmaxf(v, 0.f) : v;
    }
}
}  // namespace

int mdx_channel_affine(const float* x, const float* scale, const float* shift, float* y, int64_t batch, int channels,
                       int64_t plane, bool relu, cudaStream_t s) {
    const int64_t total = batch * channels * plane;
    if (total <= 0 || (x == y && !scale && !shift && !relu)) return ANCHA_OK;
    channel_affine_kernel<<<blocks_for(total), kThreads, 0, s>>>(x, scale, shift, y, channels, plane, total, relu);
    return check_launch("mdx_channel_affine");
}

int mdx_matmul(const float* a, const float* b, float* out, const MdxMatmul& m, cudaStream_t s) {
    const int64_t batches = m.batch[0] * m.batch[1];
    if (batches <= 0 || m.m <= 0 || m.n <= 0) return ANCHA_OK;
    if (batches > 65535 || ceil_div(m.m, 16) > 65535) return fail(ANCHA_E_UNSUPPORTED, "mdx_matmul: grid too large");
    const dim3 grid((unsigned)ceil_div(m.n, 16), (unsigned)ceil_div(m.m, 16), (unsigned)batches);
    matmul_kernel<<<grid, dim3(16, 16), 0, s>>>(a, b, out, m);
    return check_launch("mdx_matmul");
}

}  // namespace ancha
