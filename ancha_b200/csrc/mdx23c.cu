// MDX23C device kernels (declared in mdx23c.cuh). All of them are HBM-bound gathers and
// elementwise passes around the network's GEMMs:
//
// * mdx_plane_stats: f64 sum and sum of squares per NCHW plane (the instance norms of
//   mdx23c.rs:200-213 reduce over a whole (batch, channel) plane, so the statistics must be
//   complete before any element is normalised);
// * mdx_pack: norm → GELU → zero-padded patch gather into the K-major patch matrix of a
//   convolution (the B operand of out[co][pos] = W[co][k]·P[pos][k]ᵀ), over a channel
//   concatenation of two sources so the decoder's cat(up, skip) and the final cat(mix, x)
//   are never materialised. One CTA stages the normalised input rows of 32 output columns ×
//   32 channels in shared memory and writes each patch row's 32·kh·kw columns contiguously;
// * mdx_norm_act, mdx_transpose, mdx_shuffle2x2: the TDF input, the time / frequency swaps
//   of mdx23c.rs:437 and 475, and the ConvTranspose2d(2, 2) scatter (spatial.rs:128-150).
#include "mdx23c.cuh"

namespace ancha {
namespace {

constexpr int kPackCols = 32;   // output columns per CTA
constexpr int kPackChans = 32;  // channels per CTA

__global__ void plane_stats_kernel(const float* __restrict__ x, int64_t n, int splits,
                                   double2* __restrict__ stats) {
    const int64_t plane = blockIdx.x;
    const int64_t per = (n + splits - 1) / splits;
    const int64_t lo = per * blockIdx.y, hi = min(n, lo + per);
    const float* p = x + plane * n;
    double s = 0.0, q = 0.0;
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const double v = p[i];
        s += v;
        q += v * v;
    }
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
        q += __shfl_xor_sync(0xffffffffu, q, o);
    }
    __shared__ double ws[2][32];
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane == 0) { ws[0][warp] = s; ws[1][warp] = q; }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x / 32;
        s = lane < nw ? ws[0][lane] : 0.0;
        q = lane < nw ? ws[1][lane] : 0.0;
        for (int o = 16; o > 0; o >>= 1) {
            s += __shfl_xor_sync(0xffffffffu, s, o);
            q += __shfl_xor_sync(0xffffffffu, q, o);
        }
        if (lane == 0) {
            atomicAdd(&stats[plane].x, s);
            atomicAdd(&stats[plane].y, q);
        }
    }
}

// mean and 1/sqrt(biased variance + eps) of a plane of n values from its f64 sums.
__device__ __forceinline__ float2 moments(double2 st, int64_t n, float eps) {
    const double mean = st.x / (double)n;
    const double var = fmax(st.y / (double)n - mean * mean, 0.0);
    return make_float2((float)mean, (float)(1.0 / sqrt(var + (double)eps)));
}

__global__ void pack_kernel(const PackArgs a, int nchunks) {
    extern __shared__ float tile[];  // [kPackChans][kh][ncols]
    const int ctot = a.a.channels + a.b.channels;
    const int chunk = blockIdx.z % nchunks, b = blockIdx.z / nchunks;
    const int ho = blockIdx.y, wo0 = blockIdx.x * kPackCols;
    const int c0 = chunk * kPackChans, cc = min(kPackChans, ctot - c0);
    const int ncols = (kPackCols - 1) * a.sw + a.kw;
    const int hi0 = ho * a.sh - a.ph, wi0 = wo0 * a.sw - a.pw;
    const int64_t plane_n = (int64_t)a.h * a.w;
    for (int i = threadIdx.x; i < cc * a.kh * ncols; i += blockDim.x) {
        const int col = i % ncols, r = (i / ncols) % a.kh, c = c0 + i / (ncols * a.kh);
        const int hi = hi0 + r, wi = wi0 + col;
        float v = 0.f;
        if (hi >= 0 && hi < a.h && wi >= 0 && wi < a.w) {
            const PackSource& src = c < a.a.channels ? a.a : a.b;
            const int cs = c < a.a.channels ? c : c - a.a.channels;
            v = src.x[((int64_t)b * src.channels + cs) * plane_n + (int64_t)hi * a.w + wi];
            if (src.stats) {
                const float2 mr = moments(src.stats[(int64_t)b * src.channels + cs], plane_n, a.eps);
                v = (v - mr.x) * mr.y * src.gamma[cs] + src.beta[cs];
            }
            if (a.gelu) v = gelu_erf(v);
        }
        tile[i] = v;
    }
    __syncthreads();
    const int taps = a.kh * a.kw;
    const int span = cc * taps;  // patch columns this CTA writes per output position
    const int k0 = c0 * taps;
    const int ktot = ctot * taps;
    const bool last = c0 + cc == ctot;
    const int width = last ? span + (int)(a.kp - ktot) : span;  // the last chunk zero-fills the pad
    const int nwo = min(kPackCols, a.wo_n - wo0);
    for (int i = threadIdx.x; i < nwo * width; i += blockDim.x) {
        const int j = i % width, wl = i / width;
        float v = 0.f;
        if (j < span) {
            const int c = j / taps, t = j % taps, ky = t / a.kw, kx = t % a.kw;
            v = tile[(c * a.kh + ky) * ncols + wl * a.sw + kx];
        }
        const int64_t row = (int64_t)b * a.ho_n * a.wo_n + (int64_t)ho * a.wo_n + wo0 + wl;
        store_elt(a.out, row * a.kp + k0 + j, v, a.out_type);
    }
}

__global__ void norm_act_kernel(const float* __restrict__ x, int64_t total, int64_t n, int channels,
                                const double2* __restrict__ stats, const float* __restrict__ gamma,
                                const float* __restrict__ beta, float eps, bool gelu, void* out,
                                int out_type) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t plane = i / n;
        float v = x[i];
        if (stats) {
            const int c = (int)(plane % channels);
            const float2 mr = moments(stats[plane], n, eps);
            v = (v - mr.x) * mr.y * gamma[c] + beta[c];
        }
        if (gelu) v = gelu_erf(v);
        store_elt(out, i, v, out_type);
    }
}

__global__ void transpose_kernel(const float* __restrict__ x, const float* __restrict__ mul, int rows,
                                 int cols, float* __restrict__ out) {
    __shared__ float t[32][33];
    const int64_t plane = blockIdx.z;
    const float* src = x + plane * rows * (int64_t)cols;
    const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = r0 + j, c = c0 + threadIdx.x;
        if (r < rows && c < cols) t[j][threadIdx.x] = src[(int64_t)r * cols + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int c = c0 + j, r = r0 + threadIdx.x;
        if (r < rows && c < cols) {
            const int64_t o = plane * rows * (int64_t)cols + (int64_t)c * rows + r;
            out[o] = t[threadIdx.x][j] * (mul ? mul[o] : 1.f);
        }
    }
}

__global__ void shuffle2x2_kernel(const float* __restrict__ y, int channels, int h, int w,
                                  int64_t total, float* __restrict__ out, int c_total, int c_off) {
    const int ow = 2 * w, oh = 2 * h;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int ox = (int)(i % ow);
        const int oy = (int)((i / ow) % oh);
        const int c = (int)((i / ((int64_t)ow * oh)) % channels);
        const int64_t b = i / ((int64_t)ow * oh * channels);
        const int row = (c * 2 + (oy & 1)) * 2 + (ox & 1);
        const float v = y[(b * channels * 4 + row) * (int64_t)h * w + (int64_t)(oy >> 1) * w + (ox >> 1)];
        out[((b * c_total + c_off + c) * oh + oy) * (int64_t)ow + ox] = v;
    }
}

int grid_for(int64_t total) {
    return (int)std::min<int64_t>(ceil_div(total, 256), 148 * 16);
}

}  // namespace

int mdx_plane_stats(const float* x, int64_t planes, int64_t n, double2* stats, cudaStream_t s) {
    if (planes <= 0 || n <= 0) return fail(ANCHA_E_INVALID, "mdx_plane_stats: empty");
    if (planes > 0x7fffffff) return fail(ANCHA_E_UNSUPPORTED, "mdx_plane_stats: too many planes");
    ANCHA_CUDA(cudaMemsetAsync(stats, 0, planes * sizeof(double2), s));
    // Enough CTAs for the whole GPU: split long planes so every SM has work.
    const int splits = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(148 * 8, planes), ceil_div(n, 8192)));
    plane_stats_kernel<<<dim3((unsigned)planes, splits), 256, 0, s>>>(x, n, splits, stats);
    return check_launch("mdx_plane_stats");
}

int mdx_pack(const PackArgs& a, cudaStream_t s) {
    const int ctot = a.a.channels + a.b.channels;
    if (a.batch <= 0 || ctot <= 0 || a.ho_n <= 0 || a.wo_n <= 0 || a.kh < 1 || a.kw < 1 || a.kh > 3 ||
        a.kw > 3 || a.sh < 1 || a.sw < 1 || a.sh > 2 || a.sw > 2)
        return fail(ANCHA_E_INVALID, "mdx_pack: geometry");
    if (a.kp < (int64_t)ctot * a.kh * a.kw) return fail(ANCHA_E_INVALID, "mdx_pack: kp below k");
    const int nchunks = (ctot + kPackChans - 1) / kPackChans;
    if ((int64_t)a.batch * nchunks > 65535 || a.ho_n > 65535)
        return fail(ANCHA_E_UNSUPPORTED, "mdx_pack: grid too large");
    const int ncols = (kPackCols - 1) * a.sw + a.kw;
    const size_t smem = (size_t)kPackChans * a.kh * ncols * sizeof(float);
    const dim3 grid((unsigned)ceil_div(a.wo_n, kPackCols), (unsigned)a.ho_n, (unsigned)(a.batch * nchunks));
    pack_kernel<<<grid, 256, smem, s>>>(a, nchunks);
    return check_launch("mdx_pack");
}

int mdx_norm_act(const float* x, int64_t planes, int64_t n, int channels, const double2* stats,
                 const float* gamma, const float* beta, float eps, bool gelu, void* out, int out_type,
                 cudaStream_t s) {
    const int64_t total = planes * n;
    if (total <= 0) return ANCHA_OK;
    norm_act_kernel<<<grid_for(total), 256, 0, s>>>(x, total, n, channels, stats, gamma, beta, eps, gelu,
                                                    out, out_type);
    return check_launch("mdx_norm_act");
}

int mdx_transpose(const float* x, const float* mul, int64_t planes, int rows, int cols, float* out,
                  cudaStream_t s) {
    if (planes <= 0 || rows <= 0 || cols <= 0) return ANCHA_OK;
    if (planes > 65535) return fail(ANCHA_E_UNSUPPORTED, "mdx_transpose: too many planes");
    transpose_kernel<<<dim3((unsigned)ceil_div(cols, 32), (unsigned)ceil_div(rows, 32), (unsigned)planes),
                       dim3(32, 8), 0, s>>>(x, mul, rows, cols, out);
    return check_launch("mdx_transpose");
}

int mdx_shuffle2x2(const float* y, int batch, int channels, int h, int w, float* out, int c_total,
                   int c_off, cudaStream_t s) {
    const int64_t total = (int64_t)batch * channels * 4 * h * w;
    if (total <= 0) return ANCHA_OK;
    shuffle2x2_kernel<<<grid_for(total), 256, 0, s>>>(y, channels, h, w, total, out, c_total, c_off);
    return check_launch("mdx_shuffle2x2");
}

}  // namespace ancha
